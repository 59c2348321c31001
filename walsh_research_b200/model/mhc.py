"""Manifold hyper-connections and the mHCWalsh model (reference: src/model/mhc.py).

The forward of ``mHCLlamaBlock`` / ``mHCWalsh`` is the fused B200 path:

  per layer  walsh_mhc_map (RMSNorm + phi + sigmoid/Sinkhorn + pre-mix + norm)
             walsh_attn_qkv_fwd (q/k/v + RoPE + KV write) -> walsh_attn_fwd
             -> walsh_head_mixer_fwd -> walsh_hadamard_linear_fwd (wo)
             -> walsh_mhc_post
             walsh_mhc_map -> walsh_moe_fwd (router + experts + site epilogue)
             walsh_chmod_stats -> walsh_chmod_mlp -> walsh_chmod_apply
  around it  walsh_embed_gather (embedding with stream_proj folded in),
             walsh_linear_fwd (stream_merge, tied logits), walsh_rmsnorm.

The RMS of the weightless mapping norm uses eps = finfo(float32).eps, the
reference's value for float32 activations, in both activation precisions.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib, ops
from . import _prep
from .chassis import CausalSelfAttention, KVCache, RMSNorm, WalshConfig, precompute_freqs_cis, rope_tables

MAP_EPS = float(torch.finfo(torch.float32).eps)


class SinkhornKnopp(nn.Module):
    """exp then n_iter x (column, row) normalisation (src/model/mhc.py:198-229)."""

    def __init__(self, n_iter=20, eps=1e-8):
        super().__init__()
        self.n_iter = n_iter
        self.eps = eps

    def forward(self, H):
        return ops.sinkhorn(H, self.n_iter, self.eps)


class ResidualStreamMapping(nn.Module):
    """H = manifold(alpha * phi(RMSNorm(x)) + bias) (src/model/mhc.py:232-318)."""

    def __init__(self, n_embd, n_streams, mapping_type="res"):
        super().__init__()
        self.n_embd = n_embd
        self.n_streams = n_streams
        self.mapping_type = mapping_type
        self.alpha = nn.Parameter(torch.tensor(0.01))
        if mapping_type == "res":
            self.phi = nn.Linear(n_streams * n_embd, n_streams * n_streams, bias=False)
            self.bias = nn.Parameter(torch.eye(n_streams) * 2.0)
            self.sinkhorn = SinkhornKnopp(n_iter=20)
        else:
            self.phi = nn.Linear(n_streams * n_embd, n_streams, bias=False)
            self.bias = nn.Parameter(torch.zeros(1, n_streams))
        nn.init.normal_(self.phi.weight, std=0.01)

    def forward(self, x):
        """x [B, T, n*C] -> [B, T, 1, n] ('pre'/'post') or [B, T, n, n] ('res')."""
        B, T, _ = x.shape
        n, C = self.n_streams, self.n_embd
        if n != 4:
            raise NotImplementedError("the fused mapping kernel implements n_streams = 4")
        rows = {"pre": (0, 4), "post": (4, 8), "res": (8, 24)}[self.mapping_type]
        phi = torch.zeros(24, n * C, device=x.device, dtype=torch.float32)
        phi[rows[0]:rows[1]] = self.phi.weight.detach().float()
        mp = torch.zeros(28, device=x.device, dtype=torch.float32)
        slot = {"pre": 0, "post": 1, "res": 2}[self.mapping_type]
        mp[slot] = self.alpha.detach().float()
        mp[4 + rows[0]:4 + rows[1]] = self.bias.detach().float().reshape(-1)
        _, hmix = ops.mhc_map(x.reshape(B, T, n, C), phi, mp, MAP_EPS)
        h = hmix[..., rows[0]:rows[1]]
        return h.reshape(B, T, n, n) if self.mapping_type == "res" else h.reshape(B, T, 1, n)


def site_params(stream: "mHCResidualStream", dtype=torch.bfloat16):
    """phi [24, n*C], mparams [28] and phi in the 16-bit stream dtype (the
    tensor-core operand copy) of one mHC site, on the device."""
    pre, post, res = stream.H_pre, stream.H_post, stream.H_res

    def build():
        phi = torch.cat([pre.phi.weight, post.phi.weight, res.phi.weight]).detach().float().contiguous()
        phi_lp = phi.to(dtype if dtype != torch.float32 else torch.bfloat16).contiguous()
        phi_frag = ops.phi_fragments(phi_lp) if phi_lp.shape[1] % 16 == 0 else None
        dev = phi.device
        mp = torch.cat([torch.stack([pre.alpha, post.alpha, res.alpha]).detach().float().reshape(3),
                        torch.zeros(1, device=dev),
                        pre.bias.detach().float().reshape(-1), post.bias.detach().float().reshape(-1),
                        res.bias.detach().float().reshape(-1)]).contiguous()
        return phi, mp, phi_lp, phi_frag
    srcs = [pre.phi.weight, post.phi.weight, res.phi.weight, pre.alpha, post.alpha, res.alpha,
            pre.bias, post.bias, res.bias]
    return _prep.cached(stream, f"site_{dtype}", srcs, build)


class mHCResidualStream(nn.Module):
    """x' = H_res x + H_post^T F(H_pre x) (src/model/mhc.py:321-381)."""

    def __init__(self, n_embd, n_streams=4):
        super().__init__()
        self.n_embd = n_embd
        self.n_streams = n_streams
        self.H_pre = ResidualStreamMapping(n_embd, n_streams, "pre")
        self.H_post = ResidualStreamMapping(n_embd, n_streams, "post")
        self.H_res = ResidualStreamMapping(n_embd, n_streams, "res")

    def forward(self, x, layer_fn):
        phi, mp, phib, phif = site_params(self, x.dtype)
        u, hmix = ops.mhc_map(x, phi, mp, MAP_EPS, phi_lp=phib, phi_frag=phif)
        return ops.mhc_post(x, layer_fn(u), hmix)


class mHCLlamaBlock(nn.Module):
    """Block with mHC streams, MoE/SwiGLU FFN and channel modulation
    (src/model/mhc.py:451-534)."""

    def __init__(self, config, n_streams=4):
        super().__init__()
        self.n_streams = n_streams
        self.n_embd = config.n_embd
        self.attention_norm = RMSNorm(config.n_embd)
        self.ffn_norm = RMSNorm(config.n_embd)
        self.attention = CausalSelfAttention(config)
        if getattr(config, "use_moe", False):
            from .moe import HadamardMoE
            self.feed_forward = HadamardMoE(config, threshold=getattr(config, "moe_threshold", 0.1),
                                            min_experts=getattr(config, "moe_min_experts", 1),
                                            max_experts=getattr(config, "moe_max_experts", 4))
        else:
            from .cayley_dickson_cuda import SwiGLUMLP
            self.feed_forward = SwiGLUMLP(config)
        self.use_channel_mod = getattr(config, "use_channel_mod", False)
        if self.use_channel_mod:
            from .moe import HadamardChannelModulation
            self.channel_mod = HadamardChannelModulation(n_embd=config.n_embd, n_blocks=None, use_ternary=True,
                                                         residual_scale=0.5)
            self.channel_mod_norm = RMSNorm(config.n_embd)
        self.attn_stream = mHCResidualStream(config.n_embd, n_streams)
        self.ffn_stream = mHCResidualStream(config.n_embd, n_streams)

    def _w(self, p):
        return p.detach().float().contiguous()

    def forward_fused(self, x, rope_cos, rope_sin, k_cache, v_cache, start_pos: int, record_stats=True,
                      stats_out=None):
        """x [B, T, n, C] (updated in place and returned).  ``stats_out``: dict
        of buffers ("mask", "probs", "weights" [B, T, E]; "scale", "shift"
        [B*n, E]) that receive this call's router and modulation statistics;
        the caller records them (used when a batch runs in parts)."""
        B, T, n, C = x.shape
        idt = k_cache.dtype  # storage type of u, q/k/v and the attention output
        # attention site
        phi, mp, phib, phif = site_params(self.attn_stream, x.dtype)
        u, hmix = ops.mhc_map(x, phi, mp, MAP_EPS, self._w(self.attention_norm.weight), self.attention_norm.eps,
                              phi_lp=phib, u_dtype=idt, phi_frag=phif)
        self.attention.forward_site(u, rope_cos, rope_sin, k_cache, v_cache, start_pos, x, hmix)
        # ffn site
        phi, mp, phib, phif = site_params(self.ffn_stream, x.dtype)
        u, hmix = ops.mhc_map(x, phi, mp, MAP_EPS, self._w(self.ffn_norm.weight), self.ffn_norm.eps, phi_lp=phib,
                              phi_frag=phif,
                              u_dtype=idt)
        ff = self.feed_forward
        ep = self.__dict__.get("_ep")
        if ep is not None and hasattr(ff, "kernel_args") and idt != torch.float32 and C == 512:
            from .. import ep as ep_mod
            mask, probs = ep_mod.moe_site(u, x, hmix, ff, ep)
            if record_stats:
                ff._record(mask.view(B, T, -1), probs.view(B, T, -1), B * T)
        elif hasattr(ff, "kernel_args"):
            w1t, w2, g, up, d, gam, k, tc = ff.kernel_args(idt)
            rt = ff.router.routing()
            if stats_out is not None:
                ops.moe(u, w1t, w2, g, up, d, gam, k, fuse=(x, hmix, x), want_stats=True, tc=tc, routing=rt,
                        stats_out=(stats_out["mask"], stats_out["probs"], stats_out["weights"]))
            elif record_stats:
                _, mask, probs, _ = ops.moe(u, w1t, w2, g, up, d, gam, k, fuse=(x, hmix, x), want_stats=True, tc=tc,
                                            routing=rt)
                ff._record(mask, probs, B * T)
            else:
                ops.moe(u, w1t, w2, g, up, d, gam, k, fuse=(x, hmix, x), tc=tc, routing=rt)
        elif hasattr(ff, "forward_site"):
            ff.forward_site(u, x, hmix)
        else:
            ops.mhc_post(x, ff(u), hmix, out=x)
        # channel modulation over the [B*n, T, C] reinterpretation of x
        if self.use_channel_mod:
            w1, w2c, gam, temp = self.channel_mod.kernel_args()
            w1d = self.channel_mod.w1_dense() if B * n >= ops.CHMOD_MLP_TC_FROM else None
            so = stats_out or {}
            _, scale, shift = ops.chmod(x.view(B * T * n, C), T, w1, w2c, gam, temp,
                                        norm_w=self._w(self.channel_mod_norm.weight),
                                        norm_eps=self.channel_mod_norm.eps, add_input=True, out=x.view(B * T * n, C),
                                        residual_scale=self.channel_mod.residual_scale, w1_dense=w1d,
                                        scale_out=so.get("scale"), shift_out=so.get("shift"))
            if stats_out is None:
                self.channel_mod._last_scale, self.channel_mod._last_shift = scale, shift
        return x

    def forward(self, x, freqs_cis, kv_cache=None, layer_idx=0):
        B, T, n, C = x.shape
        x = x.contiguous().clone()
        cos = freqs_cis[:T].real.float().contiguous()
        sin = freqs_cis[:T].imag.float().contiguous()
        H, hd = self.attention.n_head, self.attention.head_dim
        if kv_cache is None:
            kc = torch.empty((B, H, T, hd), dtype=_lib.inner_dtype(x.dtype), device=x.device)
            vc = torch.empty_like(kc)
            start = 0
        else:
            kc, vc, start = kv_cache.k_cache[layer_idx], kv_cache.v_cache[layer_idx], kv_cache.cached_len
        return self.forward_fused(x, cos, sin, kc, vc, start)


class mHCWalsh(nn.Module):
    """Walsh with mHC residual streams (src/model/mhc.py:537-789).

    ``compute_dtype`` (float32 or bfloat16) selects the activation precision;
    a forward run under ``torch.autocast('cuda', dtype=torch.bfloat16)`` uses
    bfloat16 as well.  Parameters stay float32, as in the reference.

    In 16-bit mode every tensor-core operand is 16-bit with float32
    accumulation, and the residual stream is stored in ``stream_dtype``:
    float16 by default (8x finer rounding than bfloat16; the stream is
    bounded by the convex H_res mixing, H_post < 2 and the normalised
    channel-modulation terms), or ``torch.bfloat16`` for bfloat16's range.
    The normalised activations (u, q/k/v, attention output, SwiGLU hidden)
    are float16 in both cases."""

    def __init__(self, config, n_streams=4, gradient_checkpointing=False):
        super().__init__()
        self.config = config
        self.n_streams = n_streams
        self.gradient_checkpointing = gradient_checkpointing
        self.compute_dtype = torch.float32
        self.stream_dtype = None  # 16-bit mode stream storage: None -> float16
        if getattr(config, "hash_embeddings", False):
            from .hash_embeddings import HashEmbedding
            self.tok_embeddings = HashEmbedding(config.vocab_size, config.n_embd)
            self.output = None
        else:
            self.tok_embeddings = nn.Embedding(config.vocab_size, config.n_embd)
            self.output = nn.Linear(config.n_embd, config.vocab_size, bias=False)
            self.tok_embeddings.weight = self.output.weight
        self.stream_proj = nn.Linear(config.n_embd, n_streams * config.n_embd)
        self.layers = nn.ModuleList([mHCLlamaBlock(config, n_streams) for _ in range(config.n_layer)])
        self.stream_merge = nn.Linear(n_streams * config.n_embd, config.n_embd)
        self.norm = RMSNorm(config.n_embd)
        self.register_buffer("freqs_cis", precompute_freqs_cis(config.n_embd // config.n_head, config.block_size * 2))
        self.apply(self._init_weights)
        with torch.no_grad():
            C = config.n_embd
            self.stream_proj.weight.copy_(torch.eye(C).repeat(n_streams, 1) / math.sqrt(n_streams))
            self.stream_proj.bias.zero_()
            self.stream_merge.weight.copy_(torch.eye(C).repeat(1, n_streams) / n_streams)
            self.stream_merge.bias.zero_()

    def _init_weights(self, module):
        if isinstance(module, nn.Linear):
            torch.nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                torch.nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            torch.nn.init.normal_(module.weight, mean=0.0, std=0.02)

    # -- device-side derived weights ------------------------------------------------
    def _act_dtype(self):
        """Residual-stream storage type of this forward."""
        dt = self.compute_dtype
        if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
            dt = torch.bfloat16
        if dt == torch.float32:
            return dt
        return self.stream_dtype or torch.float16

    def embedding_matrix(self):
        """The [V, C] token embedding, tied to the output projection: the
        embedding weight, or the matrix a hash embedding represents."""
        if self.output is None:
            return self.tok_embeddings.weight_matrix()
        return self.tok_embeddings.weight

    def stream_table(self, dtype):
        """tok_embeddings folded with stream_proj: row v = stream_proj(emb[v]), [V, n*C]."""
        emb, W, b = self.embedding_matrix(), self.stream_proj.weight, self.stream_proj.bias

        def build():
            e = emb.detach().float().contiguous()
            if ops.split_eligible(e, e.shape[1]):
                t = ops.linear_split(e, *ops.split_bf16(W), b.detach())
                return t if dtype == torch.float32 else t.to(dtype)
            return ops.linear(e, W.detach().float(), b.detach(), out_dtype=dtype)
        return _prep.cached(self, f"table_{dtype}", [emb, W, b], build)

    def head_weights(self):
        """The tied output projection, float32 (logits are always computed against fp32 weights)."""
        emb = self.embedding_matrix()
        return _prep.cached(self, "emb_f32", [emb], lambda: emb.detach().float().contiguous())

    def head_weights_split(self):
        """The tied output projection as its bf16 split (w_hi, w_lo)."""
        emb = self.embedding_matrix()
        return _prep.cached(self, "emb_split", [emb], lambda: ops.split_bf16(emb))

    def head_weights_split3(self):
        """The tied output projection as [w_hi | w_lo | w_hi] bf16 [V, 3C] (linear_split_tc)."""
        emb = self.embedding_matrix()
        return _prep.cached(self, "emb_split3", [emb], lambda: ops.split3_weights(emb))

    def merge_weights_split(self):
        W = self.stream_merge.weight
        return _prep.cached(self, "merge_split", [W], lambda: ops.split_bf16(W))

    def _merge_norm(self, x, rows_last_only: bool):
        B, T, n, C = x.shape
        Wm = self.stream_merge.weight.detach().float().contiguous()
        bm = self.stream_merge.bias.detach().float().contiguous()
        nw = self.norm.weight.detach().float().contiguous()
        if rows_last_only:
            xl = x[:, T - 1]                                   # [B, n, C] strided view
            if ops.split_eligible(xl, n * C, ldx=T * n * C):
                hm = ops.linear_split(xl, *self.merge_weights_split(), bm, ldx=T * n * C, M=B)
            else:
                hm = ops.linear(xl, Wm, bm, ldx=T * n * C, M=B)    # [B, C] float32
            h = ops.rmsnorm(hm, nw, self.norm.eps, torch.float32)
            return h.view(B, 1, C)
        xf = x.view(B, T, n * C)
        if ops.split_eligible(xf, n * C):
            hm = ops.linear_split(xf, *self.merge_weights_split(), bm)
        else:
            hm = ops.linear(xf, Wm, bm)
        return ops.rmsnorm(hm, nw, self.norm.eps, torch.float32)

    def _logits(self, h):
        """h [M, C] float32 -> logits [M, V] float32 against the tied embedding."""
        if h.dtype == torch.float32 and h.shape[-1] % 8 == 0 and self.compute_dtype != torch.float32:
            # 16-bit mode: the split products on the tcgen05 tensor cores
            return ops.linear_split_tc(h, self.head_weights_split3())
        if ops.split_eligible(h, h.shape[-1]):
            return ops.linear_split(h, *self.head_weights_split())
        return ops.linear(h, self.head_weights(), None, out_dtype=torch.float32)

    # -- CUDA-graph replay of cache-free inference forwards ------------------------------
    def enable_cuda_graphs(self, enabled: bool = True):
        """Replay captured CUDA graphs for inference forwards without a KV cache
        (no targets, no hidden states, gradients off): the first call of a
        (shape, start_pos, dtype, device) runs eagerly and builds the derived
        weights, the second captures the whole forward into a graph, later calls
        copy the ids into the graph's input and replay it, one launch for the
        host instead of one per kernel.  Logits come back as a new tensor.  A
        graph is rebuilt after any parameter changes (load_state_dict, in-place
        update, ``.to()``).  Graphs hold their activations in a private memory
        pool until disabled."""
        self._graphs_on = bool(enabled)
        self.__dict__["_walsh_graphs"] = {}

    def enable_expert_parallel(self, ep=None):
        """Evaluate the MoE layers expert-parallel through ``ep`` (an
        walsh_research_b200.ep.ExpertParallel of the process group; every rank
        runs the same forward on its own tokens), or replicated again with
        None.  Applies to 16-bit forwards with n_embd = 512; others stay
        replicated.  Captured CUDA graphs are dropped."""
        for layer in self.layers:
            layer.__dict__["_ep"] = ep
        self.__dict__["_walsh_graphs"] = {}

    def set_moe_routing(self, mode: str = "topk"):
        """Expert selection of every MoE layer: "topk" (the reference's forward,
        src/model/moe.py:432-436) or "threshold" (every expert with router
        probability above config.moe_threshold, at least moe_min_experts and
        at most moe_max_experts; the rule src/model/moe.py:383-403 documents).
        Captured CUDA graphs are dropped, since they hold the rule."""
        if mode not in ("topk", "threshold"):
            raise ValueError(f"routing mode must be 'topk' or 'threshold', got {mode!r}")
        for layer in self.layers:
            ff = layer.feed_forward
            if hasattr(ff, "router"):
                ff.router.routing_mode = mode
        self.__dict__["_walsh_graphs"] = {}

    def _param_key(self):
        return tuple((p.data_ptr(), p._version) for p in self.parameters())

    def _graph_key(self, idx, start_pos):
        """Cache key of a captured forward: ids shape, start_pos, activation
        dtype, device and the experts' selection rule of every layer."""
        rule = tuple(getattr(getattr(l.feed_forward, "router", None), "routing_mode", None) for l in self.layers)
        return (tuple(idx.shape), start_pos, self._act_dtype(), idx.device, rule)

    def _graph_forward(self, idx, start_pos):
        graphs = self.__dict__.setdefault("_walsh_graphs", {})
        key = self._graph_key(idx, start_pos)
        pkey = self._param_key()
        ent = graphs.get(key)
        if ent is not None and ent["params"] != pkey:
            del graphs[key]
            ent = None
        if ent is None:
            if graphs.get(("seen",) + key) != pkey:        # first call: eager, builds derived weights
                graphs[("seen",) + key] = pkey
                return self._forward(idx, None, None, start_pos, False)
            static_idx = idx.clone()
            torch.cuda.synchronize(idx.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                logits, _ = self._forward(static_idx, None, None, start_pos, False)
            ent = {"graph": g, "idx": static_idx, "logits": logits, "err": self._last_index_error, "params": pkey}
            graphs[key] = ent
        else:
            ent["idx"].copy_(idx, non_blocking=True)
        ent["graph"].replay()
        self._last_index_error = ent["err"]
        return ent["logits"].clone(), None

    def forward(self, idx, targets=None, kv_cache=None, start_pos=0, return_hidden=False):
        if not idx.is_cuda:
            raise RuntimeError("walsh_research_b200 runs on CUDA devices only (no CPU fallback)")
        if (getattr(self, "_graphs_on", False) and kv_cache is None and targets is None and not return_hidden
                and not torch.is_grad_enabled()):
            return self._graph_forward(idx, start_pos)
        return self._forward(idx, targets, kv_cache, start_pos, return_hidden)

    def _forward(self, idx, targets, kv_cache, start_pos, return_hidden):
        B, T = idx.shape
        C, n = self.config.n_embd, self.n_streams
        dt = self._act_dtype()
        err = torch.zeros(1, dtype=torch.int32, device=idx.device)
        x = ops.embed_gather(idx, self.stream_table(dt), err).view(B, T, n, C)
        cos_all, sin_all = rope_tables(self, self.freqs_cis)
        cos, sin = cos_all[start_pos:start_pos + T], sin_all[start_pos:start_pos + T]
        idt = _lib.inner_dtype(dt)
        if kv_cache is None:
            H, hd = self.config.n_head, C // self.config.n_head
            kc = torch.empty((B, H, T, hd), dtype=idt, device=idx.device)
            vc = torch.empty_like(kc)
        elif kv_cache.dtype != idt or kv_cache.batch_size != B:
            raise ValueError(f"KV cache holds {kv_cache.batch_size} x {kv_cache.dtype}; this forward needs "
                             f"{B} x {idt} (a {dt} residual stream keeps attention in {idt})")
        elif kv_cache.cached_len + T > kv_cache.max_seq_len:
            raise ValueError("KV cache is full")
        parts = self._decode_parts(B, T, kv_cache)
        if parts > 1:
            self._layers_in_parts(x, cos, sin, kv_cache, parts)
        else:
            for l, layer in enumerate(self.layers):
                if kv_cache is not None:
                    kc, vc = kv_cache.k_cache[l], kv_cache.v_cache[l]
                    cpos = kv_cache.cached_len
                else:
                    cpos = 0
                layer.forward_fused(x, cos, sin, kc, vc, cpos)
        self._last_index_error = err
        need_all = return_hidden or targets is not None
        h_out = self._merge_norm(x, rows_last_only=not need_all)
        if targets is not None and self.output is None:
            # hash embeddings: the reference returns the chunked cross entropy and no logits
            loss = F.cross_entropy(self._logits(h_out.reshape(B * T, C)), targets.reshape(-1), ignore_index=-1)
            logits = None
        elif targets is not None:
            logits = self._logits(h_out.reshape(B * T, C)).view(B, T, -1)
            loss = F.cross_entropy(logits.view(-1, logits.size(-1)), targets.view(-1), ignore_index=-1)
        else:
            last = h_out[:, -1, :] if need_all else h_out[:, 0, :]
            logits = self._logits(last.contiguous()).view(B, 1, -1)
            loss = None
        if return_hidden:
            return logits, loss, h_out
        return logits, loss

    # Batched decode can run the batch in `decode_streams` parts, each on its
    # own CUDA stream: sequences share nothing inside the layer stack, so one
    # part's latency-bound small kernels (mapping, projections, router, MoE,
    # modulation) may run beside another part's attention, which streams the
    # KV cache.  Every kernel sees the rows it would see on the whole batch;
    # the parts join before the final norm and logits.  Off by default: at
    # B256 x ctx 1024 (Walsh-512) two parts measured 2.957 ms per step against
    # 2.972 ms whole (the attention grid fills every SM, so the small kernels
    # wait for its CTAs), for twice the launches.
    decode_streams = 1
    DECODE_PARTS_FROM = 128  # batch size from which a T <= 4 step is split

    def _decode_parts(self, B, T, kv_cache):
        if kv_cache is None or T > 4 or B < self.DECODE_PARTS_FROM or self.decode_streams < 2:
            return 1
        if torch.is_grad_enabled() or any(l.__dict__.get("_ep") is not None for l in self.layers):
            return 1
        return min(int(self.decode_streams), B)

    def _side_streams(self, dev, k):
        cache = self.__dict__.setdefault("_part_streams", {})
        key = (dev.index, k)
        if key not in cache:
            cache[key] = [torch.cuda.Stream(device=dev) for _ in range(k)]
        return cache[key]

    def _layers_in_parts(self, x, cos, sin, kv_cache, parts):
        B, T, n, C = x.shape
        E, dev = C // 32, x.device
        cpos = kv_cache.cached_len
        bounds = [B * i // parts for i in range(parts + 1)]
        # full-batch statistics buffers; each part writes its rows
        stats = []
        for layer in self.layers:
            st = {}
            if hasattr(layer.feed_forward, "kernel_args"):
                st["mask"] = torch.empty((B, T, E), dtype=torch.uint8, device=dev)
                st["probs"] = torch.empty((B, T, E), dtype=torch.float32, device=dev)
                st["weights"] = torch.empty((B, T, E), dtype=torch.float32, device=dev)
            if layer.use_channel_mod:
                st["scale"] = torch.empty((B * n, E), dtype=torch.float32, device=dev)
                st["shift"] = torch.empty((B * n, E), dtype=torch.float32, device=dev)
            stats.append(st)
        main = torch.cuda.current_stream(dev)
        side = self._side_streams(dev, parts - 1)
        for s in side:
            s.wait_stream(main)
        for l, layer in enumerate(self.layers):
            kc, vc = kv_cache.k_cache[l], kv_cache.v_cache[l]
            for p in range(parts):
                b0, b1 = bounds[p], bounds[p + 1]
                so = {k: (v[b0 * n:b1 * n] if k in ("scale", "shift") else v[b0:b1]) for k, v in stats[l].items()}
                with torch.cuda.stream(main if p == 0 else side[p - 1]):
                    layer.forward_fused(x[b0:b1], cos, sin, kc[b0:b1], vc[b0:b1], cpos, stats_out=so)
        for s in side:
            main.wait_stream(s)
        for layer, st in zip(self.layers, stats):
            if "mask" in st:
                layer.feed_forward._record(st["mask"], st["probs"], B * T)
            if "scale" in st:
                layer.channel_mod._last_scale, layer.channel_mod._last_shift = st["scale"], st["shift"]

    def check_token_ids(self):
        """Raise if the last forward saw a token id outside the vocabulary."""
        err = getattr(self, "_last_index_error", None)
        if err is not None and int(err.item()) != 0:
            raise IndexError("token id out of range in the last forward")

    @property
    def num_parameters(self):
        total = sum(p.numel() for p in self.parameters())
        return total, sum(p.numel() for p in self.parameters() if p.requires_grad)

    def get_aux_loss(self):
        aux = 0.0
        for layer in self.layers:
            if hasattr(layer.feed_forward, "get_aux_loss"):
                aux = aux + layer.feed_forward.get_aux_loss()
        return aux

    def get_moe_stats(self) -> dict:
        stats = [l.feed_forward.get_expert_stats() for l in self.layers if hasattr(l.feed_forward, "get_expert_stats")]
        if not stats:
            return {}
        E = len(stats[0]["expert_load"])
        avg = [sum(s["expert_load"][i] for s in stats) / len(stats) for i in range(E)]
        return {"expert_load": avg, "avg_experts": sum(s["avg_experts"] for s in stats) / len(stats),
                "load_balance": sum(s["load_balance"] for s in stats) / len(stats)}

    def reset_moe_stats(self):
        for layer in self.layers:
            if hasattr(layer.feed_forward, "reset_stats"):
                layer.feed_forward.reset_stats()

    def get_channel_mod_stats(self) -> dict:
        stats = [l.channel_mod.get_modulation_stats() for l in self.layers if hasattr(l, "channel_mod")]
        if not stats:
            return {}
        return {k: sum(s[k] for s in stats) / len(stats) for k in ("scale_mean", "scale_std", "shift_mean")}

    @staticmethod
    def _sample(logits, temperature, top_k, generator=None):
        """One token per row of logits [B, V]: scale by 1/temperature, keep the
        top_k largest (others to -inf) when top_k is set, softmax, one
        multinomial draw -- the reference's sampling step
        (src/model/mhc.py:767-782).  Returns [B, 1] int64 on the logits' device."""
        z = logits.float() / temperature
        if top_k is not None and top_k > 0:
            kth = torch.topk(z, min(int(top_k), z.shape[-1]), dim=-1).values[:, -1:]
            z = z.masked_fill(z < kth, float("-inf"))
        return torch.multinomial(F.softmax(z, dim=-1), num_samples=1, generator=generator)

    @torch.no_grad()
    def generate(self, idx, max_new_tokens, temperature=1.0, top_k=None, use_cache=True, generator=None):
        """Autoregressive sampling, [B, T] -> [B, T + new] token ids, with the
        reference's per-step rule (temperature, optional top-k, multinomial;
        src/model/mhc.py:753-789).

        use_cache=True (default): the prompt (its last block_size tokens) is
        prefilled once into a batched KV cache of block_size positions and each
        later step forwards only the B new tokens, as the reference's cached
        Walsh.generate does for one sequence (src/model/chassis.py:600-655);
        generation stops early once the cache is full.  use_cache=False
        re-forwards the cropped context for every token, as mHCWalsh.generate
        does in the reference.  ``generator`` seeds the draws (a
        torch.Generator on the model's device)."""
        if max_new_tokens <= 0:
            return idx
        bs = self.config.block_size
        if not use_cache:
            seq = idx
            for _ in range(max_new_tokens):
                logits, _ = self(seq[:, -bs:])
                seq = torch.cat((seq, self._sample(logits[:, -1, :], temperature, top_k, generator)), dim=1)
            return seq
        ctx = idx[:, -bs:]
        B, T = ctx.shape
        C, H = self.config.n_embd, self.config.n_head
        cache = KVCache(self.config.n_layer, bs, H, C // H, idx.device, dtype=_lib.inner_dtype(self._act_dtype()),
                        batch_size=B)
        logits, _ = self(ctx, kv_cache=cache, start_pos=0)
        cache.increment(T)
        nxt = self._sample(logits[:, -1, :], temperature, top_k, generator)
        out = [idx, nxt]
        for _ in range(max_new_tokens - 1):
            if cache.cached_len >= bs:
                break
            logits, _ = self(nxt, kv_cache=cache, start_pos=cache.cached_len)
            cache.increment(1)
            nxt = self._sample(logits[:, -1, :], temperature, top_k, generator)
            out.append(nxt)
        return torch.cat(out, dim=1)
