"""Generate the golden fixtures by running the reference's own PyTorch code.

Usage (in a container where the reference checkout is readable):

    python tests/golden/make_golden.py --ref /path/to/Walsh-Research

For every case in ``cases.py`` this builds the reference module
(src/model/*.py, unmodified), loads the deterministic parameters from
``cases.py`` into it, runs the forward pass on CPU in float32 and stores the
outputs as ``tests/golden/<case>.npz``.  Inputs and weights are not stored:
``cases.py`` regenerates them bit-identically from their seeds.

The octonion model is built with ``chassis.OctonionTernaryLinear`` pointed at
``physics.OctonionTernaryLinearRef`` (the reference's own CPU implementation;
its Triton layer cannot run without a GPU).  Both classes share parameter
names, shapes and semantics (src/model/physics.py:53-82,
src/model/cayley_dickson_cuda.py:622-668).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def _t(a):
    return torch.from_numpy(np.array(a, order="C", copy=True))


def _load(module, sd):
    missing, unexpected = module.load_state_dict({k: _t(v) for k, v in sd.items()}, strict=False)
    assert not unexpected, unexpected
    # only non-parameter buffers (H matrices, RoPE table, sign tables, tied output) may be missing
    params = {n for n, _ in module.named_parameters()}
    bad = [m for m in missing if m in params and m != "output.weight"]
    assert not bad, bad


def build_model(ref, cfg, n_streams):
    chassis = ref["chassis"]
    chassis.OctonionTernaryLinear = ref["physics"].OctonionTernaryLinearRef
    model = ref["mHCWalsh"](ref["WalshConfig"](**cfg), n_streams=n_streams)
    return model.eval()


def run_model_case(ref, name):
    cfg, n, idx, sd = cases.model_inputs(name)
    model = build_model(ref, cfg, n)
    _load(model, sd)
    layer_out, masks, probs = [], [], []

    def _record_router(m, i, o):
        masks.append(o[1].detach().numpy())
        probs.append(o[2].detach().numpy())
    def _record_layer(m, i, o):
        layer_out.append(o.detach().numpy())

    hooks = [layer.register_forward_hook(_record_layer) for layer in model.layers]
    if cfg["use_moe"]:
        for layer in model.layers:
            hooks.append(layer.feed_forward.router.register_forward_hook(_record_router))
    with torch.no_grad():
        logits, _, h = model(_t(idx), return_hidden=True)
    for hk in hooks:
        hk.remove()
    out = dict(logits=logits.numpy(), hidden=h.numpy())
    if name == "model_h512":
        out.update({f"layer{i}": a for i, a in enumerate(layer_out)})
    if masks:
        out["router_mask"] = np.stack(masks).astype(np.uint8)
        out["router_probs"] = np.stack(probs)
    return out


def run_decode_case(ref, name):
    cfg, n, toks, T0, steps, sd = cases.decode_inputs(name)
    model = build_model(ref, cfg, n)
    _load(model, sd)
    C, H = cfg["n_embd"], cfg["n_head"]
    cache = ref["KVCache"](cfg["n_layer"], cfg["block_size"], H, C // H, torch.device("cpu"), torch.float32)
    outs = []
    with torch.no_grad():
        logits, _ = model(_t(toks[:, :T0]), kv_cache=cache, start_pos=0)
        cache.increment(T0)
        outs.append(logits.numpy())
        for s in range(steps):
            logits, _ = model(_t(toks[:, T0 + s:T0 + s + 1]), kv_cache=cache, start_pos=cache.cached_len)
            cache.increment(1)
            outs.append(logits.numpy())
    return dict(logits=np.concatenate(outs, axis=1))


def run_op_case(ref, name):
    d = cases.op_case(name)
    fht, physics, moe, mhc, chassis = ref["fht_cuda"], ref["physics"], ref["moe"], ref["mhc"], ref["chassis"]
    with torch.no_grad():
        if name == "pack":
            out = {}
            for k in ("w_a", "w_b", "w_c"):
                packed = fht.pack_ternary_weights(_t(d[k]))
                out[k + "_packed"] = packed.numpy()
                back = fht.unpack_ternary_weights(packed, d[k].shape[-1]).numpy()
                assert np.array_equal(back, d[k])
            return out
        if name == "quant":
            return dict(unscaled=physics.quantize_ternary(_t(d["w_unscaled"])).numpy(),
                        scaled=moe.quantize_ternary(_t(d["w_scaled"])).numpy())
        if name.startswith("hlin_"):
            fin, fout = d["x"].shape[-1], d["weight"].shape[1] * 32
            layer = fht.HadamardLinear(fin, fout).eval()
            layer.weight.copy_(_t(d["weight"])); layer.alpha.copy_(_t(d["alpha"])); layer.beta.copy_(_t(d["beta"]))
            return dict(y=layer(_t(d["x"])).numpy())
        if name.startswith("headmix"):
            hd = d["x"].shape[-1]
            layer = fht.HadamardHeadMixerFused(hd).eval()
            layer.W.copy_(_t(d["W"])); layer.beta.copy_(_t(d["beta"]))
            return dict(y=layer(_t(d["x"])).numpy())
        if name == "sinkhorn":
            return dict(y=mhc.SinkhornKnopp()(_t(d["H"])).numpy())
        if name == "mapping":
            out = {}
            for kind in ("pre", "post", "res"):
                m = mhc.ResidualStreamMapping(512, 4, kind).eval()
                m.phi.weight.copy_(_t(d[f"{kind}_phi"])); m.alpha.copy_(_t(d[f"{kind}_alpha"]))
                m.bias.copy_(_t(d[f"{kind}_bias"]))
                out[kind] = m(_t(d["x"])).numpy()
            return out
        if name == "moe":
            cfg = ref["WalshConfig"](n_embd=512)
            m = moe.HadamardMoE(cfg, max_experts=int(d["top_k"])).eval()
            m.router.gate[0].weight.copy_(_t(d["gate0"])); m.router.gate[2].weight.copy_(_t(d["gate2"]))
            m.experts.gate_weights.copy_(_t(d["gate_w"])); m.experts.up_weights.copy_(_t(d["up_w"]))
            m.experts.down_weights.copy_(_t(d["down_w"]))
            w, mask, probs = m.router(_t(d["x"]))
            y = m(_t(d["x"]))
            return dict(y=y.numpy(), weights=w.numpy(), mask=mask.numpy().astype(np.uint8), probs=probs.numpy())
        if name == "chmod":
            m = moe.HadamardChannelModulation(512, use_ternary=True, residual_scale=0.5).eval()
            m.context_mlp[0].weight.copy_(_t(d["w0"])); m.context_mlp[2].weight.copy_(_t(d["w2"]))
            m.scale_temp.copy_(_t(d["scale_temp"]))
            return dict(y=m(_t(d["x"])).numpy())
        if name == "octo_lin":
            layer = physics.OctonionTernaryLinearRef(512, 512).eval()
            layer.weight.copy_(_t(d["weight"])); layer.beta.copy_(_t(d["beta"]))
            ys = layer(_t(d["x"]).split(64, dim=-1))
            return dict(y=torch.cat(ys, dim=-1).numpy())
        if name == "octo_headmix":
            layer = chassis.OctonionHeadMixer(16).eval()
            layer.W.copy_(_t(d["W"])); layer.beta.copy_(_t(d["beta"]))
            return dict(y=layer(_t(d["x"])).numpy())
        if name == "hash_emb":
            nt, nb, C = d["tables"].shape
            V = d["importance"].shape[0]
            m = chassis.HashEmbedding(V, C, bucket_size=nb, num_tables=nt).eval()
            for i in range(nt):
                m.emb_tables[i].weight.copy_(_t(d["tables"][i]))
            m.importance.weight.copy_(_t(d["importance"]))
            return dict(y=m(_t(d["x"])).numpy(), all_indices=m.all_indices.numpy(),
                        hash_a=m.hash_a.numpy(), hash_b=m.hash_b.numpy(),
                        all_embeddings=m._get_all_embeddings().numpy(),
                        logits=m.output_projection(_t(d["h"])).numpy(),
                        loss=np.array(m.chunked_cross_entropy(_t(d["h"]), _t(d["targets"]), chunk_size=256).item()))
    raise KeyError(name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout (contains src/model)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    torch.set_num_threads(os.cpu_count())
    from src.model import fht_cuda, physics, moe, mhc, chassis  # noqa: E402
    from src.model import WalshConfig, mHCWalsh, KVCache  # noqa: E402
    ref = dict(fht_cuda=fht_cuda, physics=physics, moe=moe, mhc=mhc, chassis=chassis,
               WalshConfig=WalshConfig, mHCWalsh=mHCWalsh, KVCache=KVCache)
    jobs = [(n, run_op_case) for n in cases.OP_CASES] + \
           [(n, run_model_case) for n in cases.MODEL_CASES] + \
           [(n, run_decode_case) for n in cases.DECODE_CASES]
    for name, fn in jobs:
        if args.only and name != args.only:
            continue
        out = fn(ref, name)
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **out)
        print(f"{name}: {', '.join(f'{k}{list(v.shape)}' for k, v in out.items())} "
              f"-> {os.path.getsize(path) / 1024:.0f} KB")


if __name__ == "__main__":
    main()
