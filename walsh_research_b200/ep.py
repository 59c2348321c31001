"""Expert parallelism of the Hadamard MoE across the GPUs of one node.

One process per GPU (torch.distributed); tokens stay sharded by batch and
every rank keeps all weights, but each rank evaluates only the experts it
owns, for the tokens of every rank.  Expert e consumes and produces only
feature block e of a token (src/model/moe.py:536-541), so the exchange is a
transpose of the [tokens x blocks] matrix:

  dispatch  rank r sends each rank j the u columns of j's experts for its
            tokens, with the routing weights (zero outside j's experts);
  experts   rank j runs its experts over the world * T received rows;
  combine   rank j returns those experts' output columns to the tokens'
            owners, who apply the mHC site epilogue to the assembled rows.

Rank j owns experts [j E/world, (j + 1) E/world).  Two transports:

  "nvlink"  the library's exchange kernels (walsh_ep_dispatch / _combine /
            _wait): 16-byte stores into the peers' buffers (CUDA IPC
            mappings) and per-source flags with bounded device waits;
  "nccl"    torch.distributed.all_to_all_single of packed column blocks,
            the fallback when peer mappings are not available.

The exchange is the only collective; routing stays local.  Every rank must
call with the same token count and in the same order (same layers, same
steps).
"""
from __future__ import annotations

import ctypes
import pickle

import torch

from . import _lib, ops
from ._lib import call, dcode, ptr, stream


class ExpertParallelError(RuntimeError):
    pass


def owned_experts(rank: int, world: int, n_experts: int):
    """(first, count) of the experts rank owns."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    return rank * per, per


class ExpertParallel:
    """Exchange buffers and transport of one process group.

    ``max_tokens``: the largest per-rank token count of a MoE call;
    ``C``: model width (E = C / 32 experts); ``dtype``: the MoE input type
    (the 16-bit normalised activations); ``timeout_s``: budget of each
    device-side wait on a peer (the failure is raised at the next
    ``check()``)."""

    def __init__(self, group=None, max_tokens: int = 65536, C: int = 512, dtype=torch.float16,
                 transport: str = "nvlink", timeout_s: float = 10.0, device=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the NVLink exchange supports up to 8 ranks")
        if transport not in ("nvlink", "nccl"):
            raise ValueError(f"transport must be 'nvlink' or 'nccl', got {transport!r}")
        self.transport = transport
        self.C, self.E, self.dtype = C, C // 32, dtype
        self.first, self.count = owned_experts(self.rank, self.world, self.E)
        self.max_tokens = max_tokens
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda" and transport == "nvlink":
            raise ValueError("the NVLink exchange needs CUDA buffers")
        self.device = dev
        W = self.world
        self.recv_u = torch.empty((W * max_tokens, C), dtype=dtype, device=dev)
        self.recv_w = torch.zeros((W * max_tokens, self.E), dtype=torch.float32, device=dev)
        self.y_full = torch.empty((max_tokens, C), dtype=dtype, device=dev)
        self.y_local = torch.empty((W * max_tokens, C), dtype=dtype, device=dev)
        self.flags = torch.zeros(2 * W, dtype=torch.int32, device=dev)
        self.counters = torch.zeros(2 * W, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        # device clock budget of a wait (SM clocks, at most ~2 GHz)
        self.timeout_cycles = int(timeout_s * 2.0e9)
        self._mapped = []
        if transport == "nvlink":
            self._map_peers()

    # -- peer mappings ------------------------------------------------------------
    def _handle(self, t):
        n = call("walsh_ipc_handle_bytes")
        buf = ctypes.create_string_buffer(n)
        off = ctypes.c_int64(0)
        call("walsh_ipc_handle", ptr(t), buf, ctypes.byref(off))
        return buf.raw, off.value

    def _map_peers(self):
        torch.cuda.synchronize()
        mine = {name: self._handle(getattr(self, name)) for name in ("recv_u", "recv_w", "y_full", "flags")}
        allh = [None] * self.world
        self.dist.all_gather_object(allh, pickle.dumps(mine), group=self.group)
        self.peer = {}
        for name in ("recv_u", "recv_w", "y_full", "flags"):
            arr = (ctypes.c_void_p * self.world)()
            for j in range(self.world):
                if j == self.rank:
                    arr[j] = ptr(getattr(self, name))
                    continue
                h, off = pickle.loads(allh[j])[name]
                p, base = ctypes.c_void_p(), ctypes.c_void_p()
                call("walsh_ipc_open", ctypes.create_string_buffer(h, len(h)), off, ctypes.byref(p),
                     ctypes.byref(base))
                arr[j] = p.value
                self._mapped.append(base.value)
            self.peer[name] = arr
        self.dist.barrier(group=self.group)

    def close(self):
        """Unmap the peers' buffers (after every rank's last exchange)."""
        if self._mapped:
            torch.cuda.synchronize()
            self.dist.barrier(group=self.group)
            for b in self._mapped:
                call("walsh_ipc_close", ctypes.c_void_p(b))
            self._mapped = []

    # -- the exchange -------------------------------------------------------------
    def check(self):
        """Raise if a device-side wait on a peer ran out (synchronises)."""
        if self.transport == "nvlink" and int(self.status.item()) != 0:
            self.status.zero_()
            raise ExpertParallelError("a peer's expert-parallel exchange did not arrive within the timeout "
                                      f"(rank {self.rank} of {self.world})")

    def _next_epoch(self):
        self.epoch = self.epoch % 0xFFFFFFF0 + 1
        return self.epoch

    def moe(self, u, weights, experts_fn):
        """Expert output y [T, C] (u's dtype) for this rank's tokens.

        u [T, C] (16-bit, the MoE input), weights float [T, E] (routing
        weights, zero outside each token's selection).  ``experts_fn(rows,
        w_rows, first, count, out)`` evaluates experts first .. first +
        count - 1 over rows [N, C] with weights [N, E] into out [N, C]."""
        T = u.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange buffers ({self.max_tokens})")
        if u.dtype != self.dtype:
            raise TypeError(f"MoE input is {u.dtype}, the exchange buffers hold {self.dtype}")
        W = self.world
        rows, wrows = self.recv_u[: W * T], self.recv_w[: W * T]
        if self.transport == "nccl":
            self._dispatch_nccl(u, weights, T)
        else:
            ep = self._next_epoch()
            call("walsh_ep_dispatch", ptr(u), dcode(u.dtype), T, self.C, ptr(weights), self.rank, W,
                 self.peer["recv_u"], self.peer["recv_w"], self.peer["flags"], ptr(self.counters),
                 ctypes.c_uint32(ep), stream())
            call("walsh_ep_wait", ptr(self.flags), 0, W, ctypes.c_uint32(ep), self.timeout_cycles, ptr(self.status),
                 stream())
        out = self.y_local[: W * T]
        experts_fn(rows, wrows, self.first, self.count, out)
        y = self.y_full[:T]
        if self.transport == "nccl":
            self._combine_nccl(out, T)
        else:
            ep = self._next_epoch()
            call("walsh_ep_combine", ptr(out), dcode(out.dtype), T, self.C, self.rank, W, self.peer["y_full"],
                 self.peer["flags"], ptr(self.counters), ctypes.c_uint32(ep), stream())
            call("walsh_ep_wait", ptr(self.flags), W, W, ctypes.c_uint32(ep), self.timeout_cycles, ptr(self.status),
                 stream())
        return y

    # -- NCCL fallback ------------------------------------------------------------
    def _cols(self, j):
        per = self.E // self.world
        return slice(j * per * 32, (j + 1) * per * 32)

    def _dispatch_nccl(self, u, weights, T):
        W, E = self.world, self.E
        per = E // W
        send_u = torch.stack([u[:, self._cols(j)] for j in range(W)])          # [W, T, cols]
        wm = weights.view(T, W, per).permute(1, 0, 2).contiguous()              # [W, T, per]
        recv_u = torch.empty_like(send_u)
        recv_w = torch.empty_like(wm)
        self.dist.all_to_all_single(recv_u, send_u, group=self.group)
        self.dist.all_to_all_single(recv_w, wm, group=self.group)
        rows = self.recv_u[: W * T].view(W, T, self.C)
        rows[:, :, self._cols(self.rank)] = recv_u
        wr = self.recv_w[: W * T].view(W, T, W, per)
        wr.zero_()
        wr[:, :, self.rank] = recv_w

    def _combine_nccl(self, out, T):
        W = self.world
        send = out.view(W, T, self.C)[:, :, self._cols(self.rank)].contiguous()   # [W (token owner), T, cols]
        recv = torch.empty_like(send)
        self.dist.all_to_all_single(recv, send, group=self.group)
        y = self.y_full[:T]
        for j in range(W):
            y[:, self._cols(j)] = recv[j]


def tc_experts(ff, dtype):
    """experts_fn of ExpertParallel.moe for a HadamardMoE layer: the tensor-core
    expert kernel restricted to the owned experts (C = 512, 16-bit)."""
    tc = ff.kernel_args(dtype)[7]
    gammas = ff.experts.packed()[3]

    def run(rows, wrows, first, count, out):
        call("walsh_moe_experts_tc_part_fwd", ptr(rows), dcode(rows.dtype), rows.shape[0], ptr(wrows), ptr(tc[5]),
             ptr(tc[4]), ptr(gammas), first, count, ptr(out), stream())
    return run


def moe_site(u, x, hmix, ff, ep: ExpertParallel, record=None):
    """The ffn site of an mHC block with expert parallelism: local routing,
    the exchange, the owned experts, and the site epilogue on this rank's
    tokens (x updated in place).  Returns (mask, probs) of the routing."""
    C = u.shape[-1]
    T = u.numel() // C
    u2 = u.reshape(T, C)
    E = C // 32
    tc = ff.kernel_args(u.dtype)[7]
    mask = torch.empty((T, E), dtype=torch.uint8, device=u.device)
    probs = torch.empty((T, E), dtype=torch.float32, device=u.device)
    weights = torch.empty((T, E), dtype=torch.float32, device=u.device)
    rt = ops.routing_struct(ff.router.routing())
    call("walsh_moe_router_tc_fwd", ptr(u2), dcode(u.dtype), T, ptr(tc[0]), ptr(tc[1]), int(ff.router.top_k),
         ptr(mask), ptr(probs), ptr(weights), rt, stream())
    y = ep.moe(u2, weights, tc_experts(ff, u.dtype))
    ops.mhc_post(x, y.view(x.shape[:-2] + (C,)), hmix, out=x)
    return mask, probs
