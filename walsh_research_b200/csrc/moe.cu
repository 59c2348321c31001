// Hadamard MoE: router + top-k + ternary SwiGLU experts (+ optional mHC site
// epilogue) in one kernel per token tile.
//
// Reference: HadamardRouter.forward (src/model/moe.py:418-447),
// FastMoEExperts.forward (src/model/moe.py:337-380), HadamardMoE.forward
// (src/model/moe.py:512-542).  The reference evaluates all E experts and
// multiplies by a routing weight that is zero outside the top-k; here only
// the top-k (token, expert) pairs are evaluated and unselected 32-wide blocks
// are written as zeros, which is the same result.
#include <math_constants.h>

#include "common.cuh"
#include "mma.cuh"
#include "tc05.cuh"
#include "tma_host.cuh"

namespace walsh {

template <int C>
struct MoeCfg {
  static constexpr int E = C / 32;
  static constexpr int HID = C / 4;
  static constexpr int TM = C >= 2048 ? 8 : 16;
  static constexpr int JPT = HID >= 256 ? HID / 256 : 1;      // router hidden units per thread
  static constexpr int TSPLIT = HID >= 256 ? 1 : 256 / HID;   // threads sharing one hidden unit
  static constexpr int TPT = TM / TSPLIT;                      // tokens per thread (router layer 1)
  static constexpr int MAXK = 8;   // largest top_k the router accepts
};

template <typename T, typename TX, int C>
__global__ void __launch_bounds__(256)
moe_kernel(const T* __restrict__ u, int64_t ntok, RouteRule rr, const float* __restrict__ w1t,
           const float* __restrict__ w2, const uint8_t* __restrict__ gp, const uint8_t* __restrict__ upp,
           const uint8_t* __restrict__ dp, const float* __restrict__ gammas, T* __restrict__ y, int fuse_post,
           const TX* x, const float* __restrict__ hmix, TX* xo, const float* __restrict__ weights_in,
           uint8_t* __restrict__ mask_out, float* __restrict__ probs_out, float* __restrict__ weights_out) {
  using M = MoeCfg<C>;
  constexpr int E = M::E, HID = M::HID, TM = M::TM;
  extern __shared__ float4 smem4[];
  float* us = reinterpret_cast<float*>(smem4);  // [TM][C]
  float* ys = us + TM * C;                        // [TM][C]
  float* hs = ys + TM * C;                        // [TM][HID]
  float* lg = hs + TM * HID;                      // [TM][E]
  float* as = lg + TM * E;                        // [8 warps][128]
  int* sel = reinterpret_cast<int*>(as + 8 * kExpertHidden);  // [TM][E] selected experts
  float* selw = reinterpret_cast<float*>(sel + TM * E);        // [TM][E] their weights
  int* nsel = reinterpret_cast<int*>(selw + TM * E);           // [TM]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = (int64_t)blockIdx.x * TM;
  const int ntile = (int)min64(TM, ntok - t0);

  for (int i = tid; i < TM * C; i += 256) {
    const int t = i / C;
    us[i] = t < ntile ? to_f(u[t0 * C + i]) : 0.f;
    ys[i] = 0.f;
  }
  __syncthreads();

  if (weights_in) {
    // externally supplied dense routing weights: evaluate every expert with w != 0
    if (tid < ntile) {
      int n = 0;
      for (int e = 0; e < E; ++e) {
        const float wv = weights_in[(t0 + tid) * E + e];
        if (wv != 0.f) { sel[tid * E + n] = e; selw[tid * E + n] = wv; ++n; }
      }
      nsel[tid] = n;
    }
  } else {
  // router layer 1: hs[t][j] = silu(sum_k us[t][k] * W1[j][k]); W1 stored transposed [C][HID]
  {
    const int jbase = (HID >= 256) ? tid : (tid % HID);
    const int tpart = (HID >= 256) ? 0 : (tid / HID);
    float acc[M::JPT][M::TPT];
#pragma unroll
    for (int a = 0; a < M::JPT; ++a)
#pragma unroll
      for (int t = 0; t < M::TPT; ++t) acc[a][t] = 0.f;
#pragma unroll 16
    for (int k = 0; k < C; ++k) {
      float w[M::JPT];
#pragma unroll
      for (int a = 0; a < M::JPT; ++a) w[a] = __ldg(w1t + (size_t)k * HID + jbase + a * 256);
#pragma unroll
      for (int t = 0; t < M::TPT; ++t) {
        const float xv = us[(tpart * M::TPT + t) * C + k];
#pragma unroll
        for (int a = 0; a < M::JPT; ++a) acc[a][t] = fmaf(w[a], xv, acc[a][t]);
      }
    }
#pragma unroll
    for (int a = 0; a < M::JPT; ++a)
#pragma unroll
      for (int t = 0; t < M::TPT; ++t) {
        const float v = acc[a][t];
        hs[(tpart * M::TPT + t) * HID + jbase + a * 256] = v / (1.0f + expf(-v));
      }
  }
  __syncthreads();

  // router layer 2: lg[t][e] = sum_j hs[t][j] * W2[e][j]
  for (int item = tid; item < TM * E; item += 256) {
    const int t = item / E, e = item - t * E;
    const float* hp = hs + t * HID;
    const float* wp = w2 + (size_t)e * HID;
    float acc = 0.f;
#pragma unroll 16
    for (int j = 0; j < HID; ++j) acc = fmaf(hp[j], __ldg(wp + j), acc);
    lg[item] = acc;
  }
  __syncthreads();

  // softmax + top-k (ties resolved to the lower expert index), one thread per token
  if (tid < ntile) {
    float* l = lg + tid * E;
    float mx = -CUDART_INF_F;
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, l[e]);
    float sum = 0.f;
    for (int e = 0; e < E; ++e) {
      const float p = expf(l[e] - mx);
      l[e] = p;
      sum += p;
    }
    for (int e = 0; e < E; ++e) l[e] = __fdiv_rn(l[e], sum);
    uint64_t chosen = 0;
    float wsum = 0.f;
    int nk = 0;
    for (int k = 0; k < rr.kmax; ++k) {
      int best = -1;
      float bv = -1.f;
      for (int e = 0; e < E; ++e)
        if (!((chosen >> e) & 1ull) && l[e] > bv) { bv = l[e]; best = e; }
      if (best < 0) {  // non-finite scores: take the lowest unchosen expert so indices stay in range
        for (int e = E - 1; e >= 0; --e)
          if (!((chosen >> e) & 1ull)) best = e;
        bv = 0.f;
      }
      if (rr.stop(k, bv)) break;
      chosen |= 1ull << best;
      sel[tid * E + k] = best;
      selw[tid * E + k] = bv;
      ++nk;
    }
    nsel[tid] = nk;
    // renormalise in ascending expert order, as (probs * mask).sum(-1) does
    for (int e = 0; e < E; ++e)
      if ((chosen >> e) & 1ull) wsum += l[e];
    wsum = fmaxf(wsum, 1e-8f);
    for (int k = 0; k < nk; ++k) selw[tid * E + k] = __fdiv_rn(selw[tid * E + k], wsum);
    const int64_t tok = t0 + tid;
    for (int e = 0; e < E; ++e) {
      const bool on = (chosen >> e) & 1ull;
      if (mask_out) mask_out[tok * E + e] = on ? 1 : 0;
      if (probs_out) probs_out[tok * E + e] = l[e];
      if (weights_out) weights_out[tok * E + e] = on ? __fdiv_rn(l[e], wsum) : 0.f;
    }
  }
  }  // router
  __syncthreads();

  if (!gp) return;  // router-only call: outputs are the optional mask/probs/weights
  // experts: one warp per selected (token, expert) pair
  const float gg = __ldg(gammas + 0), gu = __ldg(gammas + 1), gd = __ldg(gammas + 2);
  float* aw = as + warp * kExpertHidden;
  const int slots = weights_in ? E : rr.kmax;
  for (int item = warp; item < ntile * slots; item += 8) {
    const int t = item / slots, k = item - t * slots;
    if (k >= nsel[t]) continue;
    const int e = sel[t * E + k];
    const float wgt = selw[t * E + k];
    const float* ub = us + t * C + e * kBlock;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int h = lane + 32 * q;
      const uint2 gw = __ldg(reinterpret_cast<const uint2*>(gp + ((size_t)e * kExpertHidden + h) * 8));
      const uint2 uw = __ldg(reinterpret_cast<const uint2*>(upp + ((size_t)e * kExpertHidden + h) * 8));
      float ga = 0.f, ua = 0.f;
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) {
        const uint32_t gbyte = ((bb < 4 ? gw.x : gw.y) >> (8 * (bb & 3))) & 0xffu;
        const uint32_t ubyte = ((bb < 4 ? uw.x : uw.y) >> (8 * (bb & 3))) & 0xffu;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float xv = ub[bb * 4 + j];
          ga = fmaf(tern_val(gbyte, j), xv, ga);
          ua = fmaf(tern_val(ubyte, j), xv, ua);
        }
      }
      ga *= gg;
      ua *= gu;
      aw[h] = (ga / (1.0f + expf(-ga))) * ua;
    }
    __syncwarp();
    const uint4* drow = reinterpret_cast<const uint4*>(dp + ((size_t)e * kBlock + lane) * 32);
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const uint4 dw = __ldg(drow + v);
      const uint32_t words[4] = {dw.x, dw.y, dw.z, dw.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          const uint32_t byte = (words[wi] >> (8 * bb)) & 0xffu;
          const int h0 = v * 64 + wi * 16 + bb * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) acc = fmaf(tern_val(byte, j), aw[h0 + j], acc);
        }
    }
    ys[t * C + e * kBlock + lane] = acc * gd * wgt;
    __syncwarp();
  }
  __syncthreads();

  if (!fuse_post) {
    for (int i = tid; i < ntile * C; i += 256) y[t0 * C + i] = from_f<T>(ys[i]);
    return;
  }
  for (int i = tid; i < ntile * C; i += 256) {
    const int t = i / C, c = i - t * C;
    const int64_t tok = t0 + t;
    const float* hm = hmix + tok * kMapRows;
    const size_t base = (size_t)tok * 4 * C + c;
    const float x0 = to_f(x[base]), x1 = to_f(x[base + C]), x2 = to_f(x[base + 2 * C]), x3 = to_f(x[base + 3 * C]);
    const float fv = ys[i];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float* hr = hm + 8 + 4 * r;
      const float v = (((hr[0] * x0 + hr[1] * x1) + hr[2] * x2) + hr[3] * x3) + hm[4 + r] * fv;
      xo[base + (size_t)r * C] = from_f<TX>(v);
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core variant for C = 512 (E = 16, router hidden 128), u in TU = bf16
// or fp16 with weights copied to TU.
// CTA = 8 warps x 16 tokens (128 tokens).  Shared memory holds the CTA's u
// rows and, streamed with cp.async through a double buffer, the router's W1
// in 64-column chunks and then each expert's gate/up/down weights, so every
// MMA B operand comes from shared memory via ldmatrix:
//   router   h = silu(u W1^T) [16x128] -> logits = h W2^T [16x16] (h re-packed
//            from accumulators to A fragments in registers);
//   top-k    lanes 0..15 one token each (softmax, top_k, renormalise);
//   experts  all 16 experts densely: per expert and per half of the hidden
//            units, g = u_e G_e^T, v = u_e U_e^T, a = silu(gg g) (gu v),
//            y_e += a D_e^T; the routing weight (0 when not selected) and gd
//            scale y_e, then the mHC site epilogue (or a plain store) writes
//            the expert's 32 columns.
// Ternary weights are exact in bf16/fp16; the gammas are applied in fp32.
// ---------------------------------------------------------------------------
namespace moe_tc {
constexpr int C = 512, E = 16, HID = 128, NW = 8, TOK = NW * 16;
constexpr int LDU = C + 8;               // u rows
constexpr int KC = 64, LDW1 = KC + 8;    // router W1 chunk [128][KC]
constexpr int LDG = 32 + 8;              // gate/up rows [128][32]
constexpr int LDD = HID + 8;             // down rows [32][128]
constexpr int LDW2 = HID + 8;            // W2 [16][128]
constexpr int EXPERT_ELEMS = 2 * HID * LDG + 32 * LDD;  // one expert buffer (gate, up, down)
constexpr int BUF_ELEMS = EXPERT_ELEMS > 2 * 0 + HID * LDW1 ? EXPERT_ELEMS : HID * LDW1;
template <typename TU>
constexpr size_t smem_bytes() {
  return (size_t)(TOK * LDU + 2 * BUF_ELEMS + E * LDW2) * sizeof(TU) + (size_t)NW * 16 * (E + 1) * sizeof(float);
}
}  // namespace moe_tc

template <typename TU, typename TX>
__global__ void __launch_bounds__(256, 1)
moe_mma512_kernel(const TU* __restrict__ u, int64_t ntok, RouteRule rr, const TU* __restrict__ w1b,
                  const TU* __restrict__ w2b, const TU* __restrict__ gb, const TU* __restrict__ ub,
                  const TU* __restrict__ db, const float* __restrict__ gammas, TU* __restrict__ y, int fuse_post,
                  const TX* x, const float* __restrict__ hmix, TX* xo,
                  uint8_t* __restrict__ mask_out, float* __restrict__ probs_out, float* __restrict__ weights_out) {
  using namespace moe_tc;
  extern __shared__ float4 smem4[];
  TU* us = reinterpret_cast<TU*>(smem4);                   // [TOK][LDU]
  TU* buf0 = us + TOK * LDU;                               // 2 x BUF_ELEMS
  TU* w2s = buf0 + 2 * BUF_ELEMS;                          // [E][LDW2]
  float* lgs = reinterpret_cast<float*>(w2s + E * LDW2);   // [NW][16][E+1]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int64_t cta0 = (int64_t)blockIdx.x * TOK;
  const int64_t tok0 = cta0 + warp * 16;
  TU* uw = us + warp * 16 * LDU;
  float (*lg)[E + 1] = reinterpret_cast<float (*)[E + 1]>(lgs + warp * 16 * (E + 1));

  // ---- stage u rows (zero past ntok), W2, W1 chunk 0
  for (int i = tid; i < TOK * (C / 8); i += 256) {
    const int r = i / (C / 8), c = i - r * (C / 8);
    const bool in = cta0 + r < ntok;
    cp_async16(us + r * LDU + c * 8, u + (in ? (cta0 + r) * C : 0) + c * 8, in ? 16 : 0);
  }
  for (int i = tid; i < E * (HID / 8); i += 256) {
    const int r = i / (HID / 8), c = i - r * (HID / 8);
    cp_async16(w2s + r * LDW2 + c * 8, w2b + r * HID + c * 8, 16);
  }
  auto load_w1 = [&](int kc, TU* dst) {
    for (int i = tid; i < HID * (KC / 8); i += 256) {
      const int r = i / (KC / 8), c = i - r * (KC / 8);
      cp_async16(dst + r * LDW1 + c * 8, w1b + (size_t)r * C + kc * KC + c * 8, 16);
    }
  };
  load_w1(0, buf0);
  cp_async_commit();

  // ---- router layer 1: [16 x 512] x [512 x 128], W1 streamed in KC-column chunks
  float hacc[HID / 8][4];
#pragma unroll
  for (int n = 0; n < HID / 8; ++n) hacc[n][0] = hacc[n][1] = hacc[n][2] = hacc[n][3] = 0.f;
  for (int kc = 0; kc < C / KC; ++kc) {
    TU* cur = buf0 + (kc & 1) * BUF_ELEMS;
    if (kc + 1 < C / KC) load_w1(kc + 1, buf0 + ((kc + 1) & 1) * BUF_ELEMS);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < KC / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, uw + (lane & 15) * LDU + kc * KC + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int np = 0; np < HID / 16; ++np) {
        uint32_t bf[4];
        ldsm_x4(bf, cur + (np * 16 + (lane & 7) + ((lane >> 4) << 3)) * LDW1 + ks * 16 + ((lane >> 3) & 1) * 8);
        mma16<TU>(hacc[2 * np], a, bf[0], bf[1]);
        mma16<TU>(hacc[2 * np + 1], a, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  // prefetch expert 0 while the router finishes
  auto load_expert = [&](int e, TU* dst) {
    TU* gd = dst;
    TU* ud = dst + HID * LDG;
    TU* dd = dst + 2 * HID * LDG;
    for (int i = tid; i < 3 * 512; i += 256) {
      const int part = i >> 9, j = i & 511;
      if (part < 2) {  // gate / up: 128 rows x 4 chunks
        const int r = j >> 2, c = j & 3;
        const TU* src = (part == 0 ? gb : ub) + ((size_t)e * HID + r) * 32 + c * 8;
        cp_async16((part == 0 ? gd : ud) + r * LDG + c * 8, src, 16);
      } else {         // down: 32 rows x 16 chunks
        const int r = j >> 4, c = j & 15;
        cp_async16(dd + r * LDD + c * 8, db + ((size_t)e * 32 + r) * HID + c * 8, 16);
      }
    }
  };
  if (gb) load_expert(0, buf0);
  cp_async_commit();

  // ---- silu, repack as A fragments, router layer 2: [16 x 128] x [128 x 16]
  float lacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
  for (int kk = 0; kk < HID / 16; ++kk) {
    uint32_t a[4];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float* c = hacc[2 * kk + half];
      a[half * 2 + 0] = pack2<TU>(siluf_(c[0]), siluf_(c[1]));
      a[half * 2 + 1] = pack2<TU>(siluf_(c[2]), siluf_(c[3]));
    }
    uint32_t bf[4];
    ldsm_x4(bf, w2s + ((lane & 7) + ((lane >> 4) << 3)) * LDW2 + kk * 16 + ((lane >> 3) & 1) * 8);
    mma16<TU>(lacc[0], a, bf[0], bf[1]);
    mma16<TU>(lacc[1], a, bf[2], bf[3]);
  }
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    lg[g][8 * n + 2 * t4] = lacc[n][0];
    lg[g][8 * n + 2 * t4 + 1] = lacc[n][1];
    lg[g + 8][8 * n + 2 * t4] = lacc[n][2];
    lg[g + 8][8 * n + 2 * t4 + 1] = lacc[n][3];
  }
  __syncwarp();
  // ---- softmax + top-k: lane t < 16 owns token t; its lg row becomes the routing weight
  if (lane < 16) {
    float* l = lg[lane];
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, l[e]);
    float p[E], sum = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) { p[e] = expf(l[e] - mx); sum += p[e]; }
#pragma unroll
    for (int e = 0; e < E; ++e) p[e] = __fdiv_rn(p[e], sum);
    uint32_t chosen = 0;
    for (int k = 0; k < rr.kmax; ++k) {
      int best = -1;
      float bv = -1.f;
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (!((chosen >> e) & 1u) && p[e] > bv) { bv = p[e]; best = e; }
      if (best < 0)
        for (int e = E - 1; e >= 0; --e)
          if (!((chosen >> e) & 1u)) best = e;
      if (rr.stop(k, bv)) break;
      chosen |= 1u << best;
    }
    float wsum = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if ((chosen >> e) & 1u) wsum += p[e];
    wsum = fmaxf(wsum, 1e-8f);
    const int64_t tok = tok0 + lane;
    const bool in = tok < ntok;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const bool on = (chosen >> e) & 1u;
      const float w = on ? __fdiv_rn(p[e], wsum) : 0.f;
      l[e] = w;
      if (in) {
        if (mask_out) mask_out[tok * E + e] = on ? 1 : 0;
        if (probs_out) probs_out[tok * E + e] = p[e];
        if (weights_out) weights_out[tok * E + e] = w;
      }
    }
  }
  __syncwarp();
  if (!gb) {  // router-only call
    cp_async_wait<0>();
    return;
  }

  // ---- experts (weights double-buffered in shared memory).  Expert e's
  // weighted output replaces the warp's (already consumed) u block e in
  // shared memory; the site epilogue streams the rows out afterwards.
  const float gg = __ldg(gammas + 0), gu = __ldg(gammas + 1), gd = __ldg(gammas + 2);
#pragma unroll 1
  for (int e = 0; e < E; ++e) {
    const TU* cur = buf0 + (e & 1) * BUF_ELEMS;
    if (e + 1 < E) load_expert(e + 1, buf0 + ((e + 1) & 1) * BUF_ELEMS);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const TU* gs = cur;
    const TU* uss = cur + HID * LDG;
    const TU* ds = cur + 2 * HID * LDG;
    uint32_t ae[2][4];
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) ldsm_x4(ae[ks], uw + (lane & 15) * LDU + e * 32 + ks * 16 + (lane >> 4) * 8);
    float yacc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) yacc[n][0] = yacc[n][1] = yacc[n][2] = yacc[n][3] = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float ga[8][4], va[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) ga[n][0] = ga[n][1] = ga[n][2] = ga[n][3] = va[n][0] = va[n][1] = va[n][2] = va[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int row = half * 64 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int col = ks * 16 + ((lane >> 3) & 1) * 8;
          uint32_t bg[4], bu[4];
          ldsm_x4(bg, gs + row * LDG + col);
          ldsm_x4(bu, uss + row * LDG + col);
          mma16<TU>(ga[2 * np], ae[ks], bg[0], bg[1]);
          mma16<TU>(ga[2 * np + 1], ae[ks], bg[2], bg[3]);
          mma16<TU>(va[2 * np], ae[ks], bu[0], bu[1]);
          mma16<TU>(va[2 * np + 1], ae[ks], bu[2], bu[3]);
        }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // hidden units half*64 + 16 kk .. +15
        uint32_t a[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float* G = ga[2 * kk + hh];
          const float* V = va[2 * kk + hh];
          a[hh * 2 + 0] = pack2<TU>(siluf_(gg * G[0]) * (gu * V[0]), siluf_(gg * G[1]) * (gu * V[1]));
          a[hh * 2 + 1] = pack2<TU>(siluf_(gg * G[2]) * (gu * V[2]), siluf_(gg * G[3]) * (gu * V[3]));
        }
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bd[4];
          ldsm_x4(bd, ds + (np * 16 + (lane & 7) + ((lane >> 4) << 3)) * LDD + half * 64 + kk * 16 +
                          ((lane >> 3) & 1) * 8);
          mma16<TU>(yacc[2 * np], a, bd[0], bd[1]);
          mma16<TU>(yacc[2 * np + 1], a, bd[2], bd[3]);
        }
      }
    }
    const float w_lo = lg[g][e] * gd, w_hi = lg[g + 8][e] * gd;
    __syncwarp();  // every lane's ldmatrix of u block e is done before it is overwritten
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int c = e * 32 + 8 * n + 2 * t4;
      *reinterpret_cast<uint32_t*>(uw + g * LDU + c) = pack2<TU>(yacc[n][0] * w_lo, yacc[n][1] * w_lo);
      *reinterpret_cast<uint32_t*>(uw + (g + 8) * LDU + c) = pack2<TU>(yacc[n][2] * w_hi, yacc[n][3] * w_hi);
    }
    __syncthreads();  // buffer (e & 1) is refilled by the next iteration's prefetch
  }
  // ---- epilogue: 8 consecutive columns per lane, 16-byte loads and stores,
  // software-pipelined over the warp's 16 tokens (token t + 1's stream rows and
  // coefficients are loaded before token t is computed; rows are disjoint, so
  // this is safe when xo aliases x)
  if (!fuse_post) {
    for (int t = 0; t < 16; ++t) {
      const int64_t tok = tok0 + t;
      if (tok >= ntok) break;
#pragma unroll
      for (int pass = 0; pass < C / 256; ++pass) {
        const int c = pass * 256 + lane * 8;
        *reinterpret_cast<uint4*>(y + tok * C + c) = *reinterpret_cast<const uint4*>(uw + t * LDU + c);
      }
    }
    return;
  }
  constexpr int NP = C / 256;
  uint4 xq[NP][4];
  float4 hq[5];  // H_post[4] | H_res[16]
  auto load_tok = [&](int64_t tok, uint4 (&xr)[NP][4], float4 (&hr4)[5]) {
#pragma unroll
    for (int pass = 0; pass < NP; ++pass) {
      const size_t base = (size_t)tok * 4 * C + pass * 256 + lane * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j) xr[pass][j] = *reinterpret_cast<const uint4*>(x + base + (size_t)j * C);
    }
    const float4* h4 = reinterpret_cast<const float4*>(hmix + tok * kMapRows + 4);
#pragma unroll
    for (int i = 0; i < 5; ++i) hr4[i] = __ldg(h4 + i);
  };
  if (tok0 < ntok) load_tok(tok0, xq, hq);
  for (int t = 0; t < 16; ++t) {
    const int64_t tok = tok0 + t;
    if (tok >= ntok) break;
    uint4 xn[NP][4];
    float4 hn[5];
    if (t + 1 < 16 && tok + 1 < ntok) load_tok(tok + 1, xn, hn);
    const float hp[4] = {hq[0].x, hq[0].y, hq[0].z, hq[0].w};
    const float hr[16] = {hq[1].x, hq[1].y, hq[1].z, hq[1].w, hq[2].x, hq[2].y, hq[2].z, hq[2].w,
                          hq[3].x, hq[3].y, hq[3].z, hq[3].w, hq[4].x, hq[4].y, hq[4].z, hq[4].w};
#pragma unroll
    for (int pass = 0; pass < NP; ++pass) {
      const int c = pass * 256 + lane * 8;
      const uint4 yv = *reinterpret_cast<const uint4*>(uw + t * LDU + c);
      const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
      const size_t base = (size_t)tok * 4 * C + c;
      uint32_t ow[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 yf = unpack2<TU>(yw[q]);
        float2 xf[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xf[j] = unpack2<TX>((&xq[pass][j].x)[q]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float* r = hr + 4 * i;
          const float a0 = (((r[0] * xf[0].x + r[1] * xf[1].x) + r[2] * xf[2].x) + r[3] * xf[3].x) + hp[i] * yf.x;
          const float a1 = (((r[0] * xf[0].y + r[1] * xf[1].y) + r[2] * xf[2].y) + r[3] * xf[3].y) + hp[i] * yf.y;
          ow[i][q] = pack2<TX>(a0, a1);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(xo + base + (size_t)i * C) = make_uint4(ow[i][0], ow[i][1], ow[i][2], ow[i][3]);
    }
#pragma unroll
    for (int pass = 0; pass < NP; ++pass)
#pragma unroll
      for (int j = 0; j < 4; ++j) xq[pass][j] = xn[pass][j];
#pragma unroll
    for (int i = 0; i < 5; ++i) hq[i] = hn[i];
  }
}

// Router layer 2 of one token on one warp (hs: silu(hpre) in shared memory,
// lane e holds expert e), softmax, top-k (ties to the lower index) and the
// renormalisation over the selected experts in ascending order; every lane
// gets sel[k] and its routing weight selw[k] = p / sum of the selected p.
template <int C>
__device__ __forceinline__ int moe_route_warp(const float* hs, const float* __restrict__ w2, int64_t tok,
                                              RouteRule rr, int lane, int* sel, float* selw,
                                               uint8_t* __restrict__ mask_out, float* __restrict__ probs_out,
                                               float* __restrict__ weights_out) {
  constexpr int E = C / 32, HID = C / 4;
  constexpr int EL = (E + 31) / 32;  // experts per lane (1 for E = 16, 2 for E = 64)
  // router layer 2 and softmax
  float l[EL], p[EL];
#pragma unroll
  for (int q = 0; q < EL; ++q) {
    const int e = lane + 32 * q;
    float acc = 0.f;
    if (e < E) {
      const float4* wr = reinterpret_cast<const float4*>(w2 + (size_t)e * HID);
#pragma unroll 4
      for (int j4 = 0; j4 < HID / 4; ++j4) {
        const float4 w = __ldg(wr + j4);
        acc = fmaf(hs[4 * j4], w.x, acc);
        acc = fmaf(hs[4 * j4 + 1], w.y, acc);
        acc = fmaf(hs[4 * j4 + 2], w.z, acc);
        acc = fmaf(hs[4 * j4 + 3], w.w, acc);
      }
    }
    l[q] = e < E ? acc : -CUDART_INF_F;
  }
  float mx = l[0];
#pragma unroll
  for (int q = 1; q < EL; ++q) mx = fmaxf(mx, l[q]);
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < EL; ++q) {
    p[q] = (lane + 32 * q < E) ? expf(l[q] - mx) : 0.f;
    sum += p[q];
  }
  sum = warp_sum(sum);
#pragma unroll
  for (int q = 0; q < EL; ++q) p[q] = __fdiv_rn(p[q], sum);
  // top-k by warp arg-max; ties go to the lower expert index
  uint32_t chosen = 0;  // bit q: this lane's expert lane + 32 q
  int nk = 0;           // the same on every lane: the arg-max below is a butterfly
  for (int k = 0; k < rr.kmax; ++k) {
    float bv = -2.f;
    int bi = E;
#pragma unroll
    for (int q = 0; q < EL; ++q) {
      const int e = lane + 32 * q;
      const float v = (e < E && !((chosen >> q) & 1u)) ? p[q] : -1.f;
      if (v > bv) { bv = v; bi = e; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (bi >= E || bv < 0.f) {  // non-finite scores: the lowest expert not yet chosen
      bi = E;
      for (int e = E - 1; e >= 0; --e) {
        const uint32_t cb = __shfl_sync(0xffffffffu, chosen, e & 31);
        if (!((cb >> (e >> 5)) & 1u)) bi = e;
      }
      bv = -1.f;
    }
    if (rr.stop(k, bv)) break;
    sel[k] = bi;
    if ((bi & 31) == lane) chosen |= 1u << (bi >> 5);
    ++nk;
  }
  // renormalise over the selected probabilities, summed in ascending expert order
  float wsum = 0.f;
  for (int e = 0; e < E; ++e) {
    const float pe = __shfl_sync(0xffffffffu, p[e >> 5 < EL ? e >> 5 : 0], e & 31);
    const uint32_t cb = __shfl_sync(0xffffffffu, chosen, e & 31);
    if ((cb >> (e >> 5)) & 1u) wsum += pe;
  }
  wsum = fmaxf(wsum, 1e-8f);
#pragma unroll
  for (int q = 0; q < EL; ++q) {
    const int e = lane + 32 * q;
    if (e < E) {
      const bool on = (chosen >> q) & 1u;
      if (mask_out) mask_out[tok * E + e] = on ? 1 : 0;
      if (probs_out) probs_out[tok * E + e] = p[q];
      if (weights_out) weights_out[tok * E + e] = on ? __fdiv_rn(p[q], wsum) : 0.f;
    }
  }
  for (int k = 0; k < nk; ++k) {
    const int e = sel[k];
    const float pe = __shfl_sync(0xffffffffu, p[e >> 5 < EL ? e >> 5 : 0], e & 31);
    selw[k] = __fdiv_rn(pe, wsum);
  }
  return nk;
}

// One selected expert of a token on one warp (lane k holds input k of the
// expert's 32-wide block): gate/up hidden units 4 per lane, SiLU(g) v into
// the warp's scratch as[EH], down outputs 1 per lane; writes its 32 outputs
// (scaled by gd and the routing weight wgt) to ys[e * 32 + lane].
template <typename TU, int C>
__device__ __forceinline__ void moe_expert_warp(const TU* __restrict__ u, int64_t tok, int e, float wgt,
                                                const uint8_t* __restrict__ gp, const uint8_t* __restrict__ upp,
                                                const uint8_t* __restrict__ dp, const float* __restrict__ gammas,
                                                int lane, float* as, float* ys) {
  constexpr int EH = kExpertHidden;
  const float gg = __ldg(gammas + 0), gu = __ldg(gammas + 1), gd = __ldg(gammas + 2);
    const float ub = to_f(u[tok * C + e * 32 + lane]);  // lane k holds input k of the block
    float ga[4] = {0.f, 0.f, 0.f, 0.f}, ua[4] = {0.f, 0.f, 0.f, 0.f};
    uint2 gw[4], uw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int h = lane + 32 * i;
      gw[i] = __ldg(reinterpret_cast<const uint2*>(gp + ((size_t)e * EH + h) * 8));
      uw[i] = __ldg(reinterpret_cast<const uint2*>(upp + ((size_t)e * EH + h) * 8));
    }
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xv = __shfl_sync(0xffffffffu, ub, bb * 4 + j);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t gbyte = ((bb < 4 ? gw[i].x : gw[i].y) >> (8 * (bb & 3))) & 0xffu;
          const uint32_t ubyte = ((bb < 4 ? uw[i].x : uw[i].y) >> (8 * (bb & 3))) & 0xffu;
          ga[i] = fmaf(tern_val(gbyte, j), xv, ga[i]);
          ua[i] = fmaf(tern_val(ubyte, j), xv, ua[i]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float g = ga[i] * gg, v = ua[i] * gu;
      as[lane + 32 * i] = (g / (1.0f + expf(-g))) * v;
    }
    __syncwarp();
    const uint4* drow = reinterpret_cast<const uint4*>(dp + ((size_t)e * 32 + lane) * 32);
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const uint4 dw = __ldg(drow + v);
      const uint32_t words[4] = {dw.x, dw.y, dw.z, dw.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          const uint32_t byte = (words[wi] >> (8 * bb)) & 0xffu;
          const int h0 = v * 64 + wi * 16 + bb * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) acc = fmaf(tern_val(byte, j), as[h0 + j], acc);
        }
    }
    ys[e * 32 + lane] = acc * gd * wgt;
}

// ---------------------------------------------------------------------------
// Decode-sized MoE (a few hundred tokens): router layer 1 is a tcgen05 GEMM
// done by the caller (hpre = u W1^T, one row per token); this kernel runs one
// warp per token for the rest: silu, router layer 2 (lane e holds expert e),
// softmax, top-k (ties to the lower index), renormalisation over the selected
// experts in ascending order, only the k selected ternary experts (gate/up
// hidden units 4 per lane, down outputs 1 per lane), and the mHC site
// epilogue.  Weights stay in L2; per-warp scratch (silu(hpre), the expert
// hidden activations and the output row) is in shared memory.
// ---------------------------------------------------------------------------
template <typename TU, typename TX, int C>
__global__ void __launch_bounds__(256)
moe_token_kernel(const TU* __restrict__ u, const TU* __restrict__ hpre, int64_t ntok, RouteRule rr,
                 const float* __restrict__ w2, const uint8_t* __restrict__ gp, const uint8_t* __restrict__ upp,
                 const uint8_t* __restrict__ dp, const float* __restrict__ gammas, TU* __restrict__ y,
                 int fuse_post, const TX* x, const float* __restrict__ hmix, TX* xo, uint8_t* __restrict__ mask_out,
                 float* __restrict__ probs_out, float* __restrict__ weights_out) {
  constexpr int HID = C / 4, EH = kExpertHidden, PER = HID + C + EH;
  extern __shared__ float4 smem4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* hs = reinterpret_cast<float*>(smem4) + warp * PER;  // [HID]
  float* ys = hs + HID;                                        // [C]
  float* as = ys + C;                                          // [EH]
  const int64_t tok = (int64_t)blockIdx.x * 8 + warp;
  if (tok >= ntok) return;  // whole warp
  // silu of router layer 1
  for (int j = lane; j < HID; j += 32) {
    const float v = to_f(hpre[tok * HID + j]);
    hs[j] = v / (1.0f + expf(-v));
  }
  for (int c = lane; c < C; c += 32) ys[c] = 0.f;
  __syncwarp();
  int sel[8];
  float selw[8];
  const int nk = moe_route_warp<C>(hs, w2, tok, rr, lane, sel, selw, mask_out, probs_out, weights_out);
  // the selected experts
  for (int k = 0; k < nk; ++k) {
    moe_expert_warp<TU, C>(u, tok, sel[k], selw[k], gp, upp, dp, gammas, lane, as, ys);
    __syncwarp();
  }
  // output row, or the mHC site epilogue
  if (!fuse_post) {
    for (int c = lane; c < C; c += 32) y[tok * C + c] = from_f<TU>(ys[c]);
    return;
  }
  const float* hm = hmix + tok * kMapRows;
  float hp[4], hr[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) hp[i] = __ldg(hm + 4 + i);
#pragma unroll
  for (int i = 0; i < 16; ++i) hr[i] = __ldg(hm + 8 + i);
  for (int c = lane * 8; c < C; c += 256) {
    const size_t base = (size_t)tok * 4 * C + c;
    float xs[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) load8(x + base + (size_t)j * C, xs[j]);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float o[8];
#pragma unroll
      for (int e8 = 0; e8 < 8; ++e8)
        o[e8] = (((hr[4 * r] * xs[0][e8] + hr[4 * r + 1] * xs[1][e8]) + hr[4 * r + 2] * xs[2][e8]) +
                 hr[4 * r + 3] * xs[3][e8]) + hp[r] * ys[c + e8];
      store8(xo + base + (size_t)r * C, o);
    }
  }
}

// Decode MoE with the selected experts spread over warps: CTA = one token,
// 8 warps.  Warp 0 routes (moe_route_warp); warp k < top_k then runs the
// token's k-th selected expert (an expert writes only its own 32-column block
// of the output row, so no two warps write the same column and the row equals
// moe_token_kernel's); all 256 threads finish with the output row or the mHC
// site epilogue, one (8-column chunk, output stream) pair per thread.  The
// token's latency is the router plus one expert instead of the router plus
// top_k experts in sequence.
template <typename TU, typename TX, int C>
__global__ void __launch_bounds__(256)
moe_token_split_kernel(const TU* __restrict__ u, const TU* __restrict__ hpre, int64_t ntok, RouteRule rr,
                       const float* __restrict__ w2, const uint8_t* __restrict__ gp, const uint8_t* __restrict__ upp,
                       const uint8_t* __restrict__ dp, const float* __restrict__ gammas, TU* __restrict__ y,
                       int fuse_post, const TX* x, const float* __restrict__ hmix, TX* xo,
                       uint8_t* __restrict__ mask_out, float* __restrict__ probs_out,
                       float* __restrict__ weights_out) {
  constexpr int HID = C / 4, EH = kExpertHidden;
  extern __shared__ float4 smem4[];
  float* hs = reinterpret_cast<float*>(smem4);  // [HID]
  float* ys = hs + HID;                         // [C]
  float* as = ys + C;                           // [8][EH]
  __shared__ int s_sel[8];
  __shared__ float s_w[8];
  __shared__ int s_nk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok = blockIdx.x;
  for (int j = threadIdx.x; j < HID; j += 256) {
    const float v = to_f(hpre[tok * HID + j]);
    hs[j] = v / (1.0f + expf(-v));
  }
  for (int c = threadIdx.x; c < C; c += 256) ys[c] = 0.f;
  __syncthreads();
  if (warp == 0) {
    int sel[8];
    float selw[8];
    const int nk = moe_route_warp<C>(hs, w2, tok, rr, lane, sel, selw, mask_out, probs_out, weights_out);
    if (lane == 0) {
      for (int k = 0; k < nk; ++k) {
        s_sel[k] = sel[k];
        s_w[k] = selw[k];
      }
      s_nk = nk;
    }
  }
  __syncthreads();
  if (warp < s_nk) moe_expert_warp<TU, C>(u, tok, s_sel[warp], s_w[warp], gp, upp, dp, gammas, lane, as + warp * EH, ys);
  __syncthreads();
  if (!fuse_post) {
    for (int c = threadIdx.x; c < C; c += 256) y[tok * C + c] = from_f<TU>(ys[c]);
    return;
  }
  const float* hm = hmix + tok * kMapRows;
  for (int i = threadIdx.x; i < (C / 8) * 4; i += 256) {
    const int r = i & 3, c = (i >> 2) * 8;
    const size_t base = (size_t)tok * 4 * C + c;
    const float h0 = __ldg(hm + 8 + 4 * r), h1 = __ldg(hm + 9 + 4 * r), h2 = __ldg(hm + 10 + 4 * r),
                h3 = __ldg(hm + 11 + 4 * r), hp = __ldg(hm + 4 + r);
    float xs[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) load8(x + base + (size_t)j * C, xs[j]);
    float o[8];
#pragma unroll
    for (int e8 = 0; e8 < 8; ++e8)
      o[e8] = (((h0 * xs[0][e8] + h1 * xs[1][e8]) + h2 * xs[2][e8]) + h3 * xs[3][e8]) + hp * ys[c + e8];
    store8(xo + base + (size_t)r * C, o);
  }
}

template <typename TU, typename TX, int C>
static int launch_moe_token(const void* u, const void* hpre, int64_t ntok, RouteRule rr, const float* w2,
                            const uint8_t* gp, const uint8_t* upp, const uint8_t* dp, const float* gammas, void* y,
                            int fuse_post, const void* x, const float* hmix, void* xo, uint8_t* mask_out,
                            float* probs_out, float* weights_out, cudaStream_t s) {
  if (rr.kmax <= 8) {
    const int smem2 = (C / 4 + C + 8 * kExpertHidden) * (int)sizeof(float);
    auto k2 = moe_token_split_kernel<TU, TX, C>;
    if (smem2 > 48 * 1024 &&
        cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2) != cudaSuccess)
      return launch_status();
    k2<<<(unsigned)ntok, 256, smem2, s>>>((const TU*)u, (const TU*)hpre, ntok, rr, w2, gp, upp, dp, gammas,
                                          (TU*)y, fuse_post, (const TX*)x, hmix, (TX*)xo, mask_out, probs_out,
                                          weights_out);
    return launch_status();
  }
  constexpr int PER = C / 4 + C + kExpertHidden;
  const int smem = 8 * PER * (int)sizeof(float);
  auto kern = moe_token_kernel<TU, TX, C>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status();
  kern<<<(unsigned)((ntok + 7) / 8), 256, smem, s>>>((const TU*)u, (const TU*)hpre, ntok, rr, w2, gp, upp, dp,
                                                     gammas, (TU*)y, fuse_post, (const TX*)x, hmix, (TX*)xo,
                                                     mask_out, probs_out, weights_out);
  return launch_status();
}

template <typename T, typename TX, int C>
static int launch_moe(const void* u, int64_t ntok, RouteRule rr, const float* w1t, const float* w2, const uint8_t* gp,
                      const uint8_t* upp, const uint8_t* dp, const float* gammas, void* y, int fuse_post,
                      const void* x, const float* hmix, void* xo, const float* weights_in, uint8_t* mask_out,
                      float* probs_out, float* weights_out, cudaStream_t s) {
  using M = MoeCfg<C>;
  const size_t smem = (2 * M::TM * C + M::TM * M::HID + M::TM * M::E + 8 * kExpertHidden) * sizeof(float) +
                      M::TM * M::E * (sizeof(int) + sizeof(float)) + M::TM * sizeof(int);
  auto kern = moe_kernel<T, TX, C>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (ntok + M::TM - 1) / M::TM;
  kern<<<(unsigned)grid, 256, smem, s>>>((const T*)u, ntok, rr, w1t, w2, gp, upp, dp, gammas, (T*)y, fuse_post,
                                         (const TX*)x, hmix, (TX*)xo, weights_in, mask_out, probs_out, weights_out);
  return launch_status();
}

template <typename TU, typename TX>
static int launch_moe_mma(const void* u, int64_t ntok, RouteRule rr, const walsh_moe_tc_weights* tc, bool experts,
                          const float* gammas, void* y, int fuse_post, const void* x, const float* hmix, void* xo,
                          uint8_t* mask_out, float* probs_out, float* weights_out, cudaStream_t s) {
  const unsigned grid = (unsigned)((ntok + moe_tc::TOK - 1) / moe_tc::TOK);
  const int smem = (int)moe_tc::smem_bytes<TU>();
  if (cudaFuncSetAttribute(moe_mma512_kernel<TU, TX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return WALSH_ERR_LAUNCH;
  moe_mma512_kernel<TU, TX><<<grid, 256, smem, s>>>(
      (const TU*)u, ntok, rr, (const TU*)tc->w1, (const TU*)tc->w2, experts ? (const TU*)tc->gate : nullptr,
      (const TU*)tc->up, (const TU*)tc->down, gammas, (TU*)y, fuse_post, (const TX*)x, hmix, (TX*)xo, mask_out,
      probs_out, weights_out);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Prefill MoE experts on the 5th-generation tensor cores (C = 512, E = 16
// experts on 32-wide Hadamard blocks, hidden 128; routing weights come from
// the router GEMM).  Persistent CTAs take (128-token tile, quarter of 4
// experts) units round-robin.  Per expert
// pair p one TMA stage brings u[:, 64p .. 64p + 63] (both experts' input
// blocks), the pair's gate/up rows packed side by side ([gate 128 | up 128
// rows] x [32 inputs of expert 2p | 32 of 2p + 1]) and the two experts' down
// rows; an expert's k-slice is selected by advancing the operand descriptors
// 64 bytes.  Per expert:
//   MMA1   D1[128 x 256] = u_e [gate_e | up_e]^T           (tensor memory 0..255)
//   SwiGLU warps 2-5, thread per token row, all 128 hidden units:
//          h = silu(gg g) (gu v) rounded to TU into a 128B-swizzled h tile
//   MMA2   Yq[:, 32 (e % 4) ..] = h down_e^T   (tensor memory 256.., two quarters of 4 experts)
// Warps 6-9 meanwhile take the previous quarter: each expert's 32 columns
// scaled by routing weight x gd, rounded to TU (as the expert output is),
// and the mHC site update of those columns (or y stored), 32 x 32 blocks
// staged through shared memory so that four lanes cover one token row, the
// next rows in flight (site_block).  So the MUFU-bound SwiGLU of quarter
// j + 1 overlaps the HBM-bound site update of quarter j.  Warp 0 issues TMA,
// warp 1 owns tensor memory and issues the MMAs.  Every wait is bounded; a
// wait that runs out sets g_moe_tc05_error.
// Replaces FastMoEExperts.forward + the site mix (src/model/moe.py:306-380,
// src/model/mhc.py site update).
// ---------------------------------------------------------------------------
// probe hook (slot, index): no code unless a profiling build defines it
#ifndef MOE_TC_TRACE
#define MOE_TC_TRACE(slot, idx)
#endif

namespace moe_tc5 {
constexpr int C = 512, E = 16, HID = 128, TOK = 128, NPAIR = 8;
constexpr int U_BYTES = TOK * 128;          // 128 rows x 64 columns
constexpr int G_BYTES = 256 * 128;          // 256 rows x 64 columns
constexpr int D_ATOM = 32 * 128;            // 32 rows x 64 columns
constexpr int D_EXP = 2 * D_ATOM;           // one expert's down rows (hidden 0..63 | 64..127)
constexpr int STAGE = U_BYTES + G_BYTES + 2 * D_EXP;
constexpr int NSTAGE = 2;
constexpr int H_ATOM = TOK * 128;
// site ring of one worker warp: per slot 8 rows x (4 streams x 32 columns of x,
// H_post | H_res, the 4 routing weights around the pass's expert)
constexpr int XS = 8 * 4 * 64, HS = 8 * 80, WS = 8 * 16, SLOT = XS + HS + WS, DEPTH = 4, RING = DEPTH * SLOT;
constexpr int OFF_H = NSTAGE * STAGE;
constexpr int OFF_YS = OFF_H + 2 * H_ATOM;     // 4 site warps x 32 x 32 floats
constexpr int OFF_RING = OFF_YS + 4 * 4096;
constexpr int OFF_BAR = OFF_RING + 4 * RING;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int NTHREADS = 320;
constexpr uint32_t TMEM_COLS = 512, COL_D1 = 0, COL_Y = 256;  // Y: two 128-column quarters (4 experts each)
__device__ __forceinline__ uint32_t sw_off(int r, int chunk) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4));
}
}  // namespace moe_tc5

__device__ int g_moe_tc05_error;

// One pass of the site update (8 rows x 32 columns = expert ex0 + step / 4)
// into ring slot `slot`: the rows' 4 stream segments, mixing coefficients
// and routing weights, by cp.async (rows past ntok are zero-filled).
template <typename TX>
__device__ __forceinline__ void site_prefetch(int64_t mw, int ex0, int step, int slot, int lane, unsigned char* ring,
                                              int64_t ntok, const float* rw, const TX* x, const float* hmix) {
  using namespace moe_tc5;
  const int k = step >> 2, p = step & 3, rq = lane >> 2, cq = lane & 3;
  unsigned char* sl = ring + slot * SLOT;
  const int64_t m = mw + p * 8 + rq;
  const bool in = m < ntok;
  const int64_t mm = in ? m : 0;
  if (x) {
    const TX* src = x + (size_t)mm * 4 * C + (ex0 + k) * 32 + cq * 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) cp_async16(sl + (rq * 4 + j) * 64 + cq * 16, src + (size_t)j * C, in ? 16 : 0);
    const float* hm = hmix + mm * kMapRows + 4;
    cp_async16(sl + XS + rq * 80 + cq * 16, hm + 4 * cq, in ? 16 : 0);
    if (cq == 0) cp_async16(sl + XS + rq * 80 + 64, hm + 16, in ? 16 : 0);
  }
  if (cq == 0) cp_async16(sl + XS + HS + rq * 16, rw + mm * E + ((ex0 + k) & ~3), in ? 16 : 0);
}

// Site update (or y store) of one worker warp after 8 experts: rows mw ..
// mw + 31 (its tensor-memory lane quarter), the 4 experts ex0 .. ex0 + 3 whose
// outputs sit in tensor memory at tacc (32 columns each).  Per expert the 32
// x 32 fp32 block is staged through the warp's 4 KB of the (idle) h tile
// (16-byte chunks XOR-swizzled by row), then 4 passes of 8 rows with four
// lanes per row (8 columns each); the next pass's rows are in flight while a
// pass is mixed.  y = D2 w gd rounded to TU, then
// x_o = H_res x + H_post y (or y stored).
template <typename TU, typename TX>
__device__ __forceinline__ void site_block(int64_t mw, int ex0, uint32_t tacc, int lane, float* ys,
                                           unsigned char* ring, int64_t ntok, const float* rw, float gd, TU* y,
                                           int fuse_post, const TX* x, const float* hmix, TX* xo) {
  using namespace moe_tc5;
  const int rq = lane >> 2, cq = lane & 3;
  const TX* xs = fuse_post ? x : nullptr;
#pragma unroll
  for (int k = 0; k < DEPTH - 1; ++k) {
    site_prefetch<TX>(mw, ex0, k, k, lane, ring, ntok, rw, xs, hmix);
    cp_async_commit();
  }
#pragma unroll 1
  for (int step = 0; step < 16; ++step) {
    const int k = step >> 2, p = step & 3, ex = ex0 + k;
    if (p == 0) {
      float v[32];
      tc05::tmem_ld32(tacc + (uint32_t)(32 * k), v);
      __syncwarp();  // the previous expert's staged rows are fully read
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4*>(ys + lane * 32 + 4 * (i ^ (lane & 7))) =
            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    cp_async_wait<DEPTH - 2>();
    __syncwarp();
    const int rr = p * 8 + rq;
    const int64_t m = mw + rr;
    const unsigned char* sl = ring + (step % DEPTH) * SLOT;
    if (m < ntok) {
      const float wgt = reinterpret_cast<const float*>(sl + XS + HS + rq * 16)[ex & 3] * gd;
      const float4 y0 = *reinterpret_cast<const float4*>(ys + rr * 32 + 4 * ((2 * cq) ^ (rr & 7)));
      const float4 y1 = *reinterpret_cast<const float4*>(ys + rr * 32 + 4 * ((2 * cq + 1) ^ (rr & 7)));
      float yf[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
      uint32_t yt[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        yt[i] = pack2<TU>(yf[2 * i] * wgt, yf[2 * i + 1] * wgt);
        const float2 back = unpack2<TU>(yt[i]);
        yf[2 * i] = back.x;
        yf[2 * i + 1] = back.y;
      }
      const int col = ex * 32 + cq * 8;
      if (!fuse_post) {
        *reinterpret_cast<uint4*>(y + m * C + col) = make_uint4(yt[0], yt[1], yt[2], yt[3]);
      } else {
        float h[20];
#pragma unroll
        for (int i = 0; i < 5; ++i) {
          const float4 hv = *reinterpret_cast<const float4*>(sl + XS + rq * 80 + 16 * i);
          h[4 * i] = hv.x;
          h[4 * i + 1] = hv.y;
          h[4 * i + 2] = hv.z;
          h[4 * i + 3] = hv.w;
        }
        float xf[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          unpack8(*reinterpret_cast<const uint4*>(sl + (rq * 4 + j) * 64 + cq * 16), xf[j], (const TX*)nullptr);
        const size_t base = (size_t)m * 4 * C + col;
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const float* hr = h + 4 + 4 * o;
          const uint64_t h0 = f2_dup(hr[0]), h1 = f2_dup(hr[1]), h2 = f2_dup(hr[2]), h3 = f2_dup(hr[3]),
                         hpo = f2_dup(h[o]);
          uint32_t ow[4];
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            // (((H0 x0 + H1 x1) + H2 x2) + H3 x3) + H_post y, two columns per instruction
            uint64_t a = f2_mul(h0, f2_pack(xf[0][i], xf[0][i + 1]));
            a = f2_fma(h1, f2_pack(xf[1][i], xf[1][i + 1]), a);
            a = f2_fma(h2, f2_pack(xf[2][i], xf[2][i + 1]), a);
            a = f2_fma(h3, f2_pack(xf[3][i], xf[3][i + 1]), a);
            a = f2_fma(hpo, f2_pack(yf[i], yf[i + 1]), a);
            ow[i >> 1] = pack2<TX>(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)(a >> 32)));
          }
          *reinterpret_cast<uint4*>(xo + base + (size_t)o * C) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
    }
    __syncwarp();  // the slot of this step is free: refill it with step + DEPTH - 1
    if (step + DEPTH - 1 < 16)
      site_prefetch<TX>(mw, ex0, step + DEPTH - 1, (step + DEPTH - 1) % DEPTH, lane, ring, ntok, rw, xs, hmix);
    cp_async_commit();
  }
  cp_async_wait<0>();
}

template <typename TU, typename TX>
__global__ void __launch_bounds__(moe_tc5::NTHREADS, 1)
moe_experts_tc05_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_g,
                        const __grid_constant__ CUtensorMap tm_d, int64_t ntok, const float* __restrict__ rw,
                        const float* __restrict__ gammas, TU* __restrict__ y, int fuse_post, const TX* x,
                        const float* __restrict__ hmix, TX* xo, int q0, int nq) {
  using namespace moe_tc5;
  using namespace tc05;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full = bars;          // [2] stage loaded (TMA)
  uint64_t* empty = bars + 2;     // [2] stage consumed (MMA commit)
  uint64_t* d1_full = bars + 4;   // MMA1 done (commit)
  uint64_t* d1_empty = bars + 5;  // D1 read by the 4 SwiGLU warps
  uint64_t* h_full = bars + 6;    // h tile written by the 4 SwiGLU warps
  uint64_t* h_empty = bars + 7;   // MMA2 done with h (commit)
  uint64_t* y_full = bars + 8;    // [2] a quarter's 4 MMA2s done (commit)
  uint64_t* y_empty = bars + 10;  // [2] a quarter read by the 4 site warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // work unit = (128-token tile, quarter of 4 experts): the quarters of a tile
  // are independent (expert e reads u columns 32e .. 32e + 31 and writes only
  // those columns of the streams), so the persistent CTAs take units
  // round-robin -- 4x finer than whole tiles, which evens out the last round.
  // Only quarters q0 .. q0 + nq - 1 are evaluated (all four by default; an
  // expert-parallel rank takes the quarters of the experts it owns): unit un
  // is tile un / nq, quarter q0 + un % nq.
  const int64_t units = (ntok + TOK - 1) / TOK * nq;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&y_full[i], 1);
      mbar_init(&y_empty[i], 4);
    }
    mbar_init(d1_full, 1);
    mbar_init(d1_empty, 4);
    mbar_init(h_full, 4);
    mbar_init(h_empty, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tm_u);
    prefetch_tensormap(&tm_g);
    prefetch_tensormap(&tm_d);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int64_t g = 0;  // expert pairs loaded by this CTA
      for (int64_t un = blockIdx.x; un < units && !*abort_flag; un += gridDim.x) {
        const int64_t t = un / nq;
        const int qu = q0 + (int)(un % nq);
        for (int p = 2 * qu; p < 2 * qu + 2; ++p, ++g) {
          const int st = (int)(g & 1);
          if (g >= 2 && !mbar_wait_sleep(&empty[st], (uint32_t)(((g >> 1) - 1) & 1))) {
            *abort_flag = 1;
            break;
          }
          unsigned char* sb = smem + st * STAGE;
          mbar_arrive_expect_tx(&full[st], STAGE);
          tma_load_2d(sb, &tm_u, &full[st], 64 * p, (int)(t * TOK));
          tma_load_2d(sb + U_BYTES, &tm_g, &full[st], 0, 256 * p);
#pragma unroll
          for (int ee = 0; ee < 2; ++ee)
#pragma unroll
            for (int a = 0; a < 2; ++a)
              tma_load_2d(sb + U_BYTES + G_BYTES + ee * D_EXP + a * D_ATOM, &tm_d, &full[st], 64 * a,
                          32 * (2 * p + ee));
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC1 = idesc_f16(std::is_same<TU, __nv_bfloat16>::value, 128, 256);
      constexpr uint32_t IDESC2 = idesc_f16(std::is_same<TU, __nv_bfloat16>::value, 128, 32);
      // iteration ge: MMA1 of expert ge (as soon as D1 is free), then MMA2 of
      // expert ge - 1 (once its h tile is written); expert ge of this CTA is
      // expert ge % 4 of its unit ge / 4, pair ge / 2 in stage (ge / 2) % 2
      const int64_t total = ((units - blockIdx.x + gridDim.x - 1) / gridDim.x) * 4;
      bool ok = true;
      const uint64_t dH = sw128_desc(smem_u32(smem + OFF_H));
      for (int64_t ge = 0; ge <= total && ok; ++ge) {
        if (ge < total) {
          const int64_t pr = ge >> 1;
          const int odd = (int)(ge & 1), st = (int)(pr & 1);
          if (!odd) ok = mbar_wait_sleep(&full[st], (uint32_t)((pr >> 1) & 1));
          if (ok && ge > 0) ok = mbar_wait_sleep(d1_empty, (uint32_t)((ge - 1) & 1));
          if (!ok) break;
          fence_after_sync();
          const uint32_t sb = smem_u32(smem + st * STAGE);
          const uint64_t dU = sw128_desc(sb), dG = sw128_desc(sb + U_BYTES);
#pragma unroll
          for (int k = 0; k < 2; ++k)
            umma_f16(tmem + COL_D1, dU + 4 * odd + 2 * k, dG + 4 * odd + 2 * k, IDESC1, k != 0);
          umma_commit(d1_full);
          MOE_TC_TRACE(0, (int)(ge & 15));
        }
        if (ge > 0) {
          const int64_t g2 = ge - 1, pr = g2 >> 1, gq = g2 >> 2;
          const int odd = (int)(g2 & 1), st = (int)(pr & 1), yb = (int)(gq & 1), e4 = (int)(g2 & 3);
          ok = mbar_wait_sleep(h_full, (uint32_t)(g2 & 1));
          if (ok && e4 == 0 && gq >= 2) ok = mbar_wait_sleep(&y_empty[yb], (uint32_t)(((gq >> 1) - 1) & 1));
          if (!ok) break;
          fence_after_sync();
          const uint64_t dD = sw128_desc(smem_u32(smem + st * STAGE) + U_BYTES + G_BYTES + odd * D_EXP);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tmem + COL_Y + 128 * yb + 32 * e4, dH + (kk >> 2) * (H_ATOM >> 4) + 2 * (kk & 3),
                     dD + (kk >> 2) * (D_ATOM >> 4) + 2 * (kk & 3), IDESC2, kk != 0);
          umma_commit(h_empty);
          MOE_TC_TRACE(1, (int)(g2 & 15));
          if (e4 == 3) umma_commit(&y_full[yb]);
          if (odd) umma_commit(&empty[st]);
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 6) {
    // ---- SwiGLU warps 2-5: tensor-memory lanes 32 (warp % 4) .., thread = token row ----
    const int q = warp & 3;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    const float gg = __ldg(gammas), gu = __ldg(gammas + 1);
    // h = SiLU(gg g) (gu v) = g v gg gu / (1 + 2^(-gg log2(e) g)): two MUFU
    // operations per value, the rest on float pairs
    const uint64_t cexp = f2_dup(-gg * 1.4426950408889634f), cgu = f2_dup(gg * gu), one2 = f2_dup(1.0f);
    const uint32_t sH = smem_u32(smem + OFF_H);
    const int r = q * 32 + lane;
    int64_t ge = 0;
    bool ok = true;
    for (int64_t un = blockIdx.x; un < units && ok; un += gridDim.x) {
      const int qu = q0 + (int)(un % nq);
      for (int e = 4 * qu; e < 4 * qu + 4 && ok; ++e, ++ge) {
        if (!__all_sync(0xffffffffu, mbar_wait(d1_full, (uint32_t)(ge & 1)))) {
          ok = false;
          break;
        }
        fence_after_sync();
        MOE_TC_TRACE(2, e);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // hidden units 32 c .. 32 c + 31
          float gv[32], uv[32];
          tmem_ld32_nowait(tl + COL_D1 + 32 * c, gv);
          tmem_ld32_nowait(tl + COL_D1 + 128 + 32 * c, uv);
          tmem_wait_ld();
          if (c == 3) {  // D1 fully read: the next expert's MMA1 may start
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(d1_empty);
          }
          uint32_t a[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint64_t g2 = f2_pack(gv[2 * i], gv[2 * i + 1]);
            const uint64_t t = f2_mul(g2, cexp);
            const uint64_t d = f2_fma(f2_pack(ex2_f32(f2_lo(t)), ex2_f32(f2_hi(t))), one2, one2);
            const uint64_t hs = f2_mul(f2_mul(g2, f2_pack(rcp_f32(f2_lo(d)), rcp_f32(f2_hi(d)))),
                                       f2_mul(f2_pack(uv[2 * i], uv[2 * i + 1]), cgu));
            a[i] = pack2<TU>(f2_lo(hs), f2_hi(hs));
          }
          if (c == 0 && ge > 0 && !__all_sync(0xffffffffu, mbar_wait(h_empty, (uint32_t)((ge - 1) & 1)))) {
            ok = false;
            break;
          }
          const uint32_t at = sH + (c >> 1) * H_ATOM;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(at + sw_off(r, 4 * (c & 1) + k)),
                         "r"(a[4 * k]), "r"(a[4 * k + 1]), "r"(a[4 * k + 2]), "r"(a[4 * k + 3])
                         : "memory");
        }
        if (!ok) break;
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(h_full);
        MOE_TC_TRACE(3, e);
      }
    }
    if (!ok) *abort_flag = 1;
  } else {
    // ---- site warps 6-9: rows 32 (warp % 4) .., one quarter (4 experts) at a time ----
    const int q = warp & 3;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    const float gd = __ldg(gammas + 2);
    float* ys = reinterpret_cast<float*>(smem + OFF_YS + (warp - 6) * 4096);
    unsigned char* ring = smem + OFF_RING + (warp - 6) * RING;
    int64_t gq = 0;
    bool ok = true;
    for (int64_t un = blockIdx.x; un < units && ok; un += gridDim.x, ++gq) {
      const int64_t t = un / nq;
      const int qt = q0 + (int)(un % nq), yb = (int)(gq & 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&y_full[yb], (uint32_t)((gq >> 1) & 1)))) {
        ok = false;
        break;
      }
      fence_after_sync();
      MOE_TC_TRACE(4, 4 * qt);
      site_block<TU, TX>(t * TOK + q * 32, 4 * qt, tl + COL_Y + 128 * yb, lane, ys, ring, ntok, rw, gd, y,
                         fuse_post, x, hmix, xo);
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&y_empty[yb]);
      MOE_TC_TRACE(5, 4 * qt);
    }
    if (!ok) *abort_flag = 1;
  }
  __syncwarp();
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_moe_tc05_error, (int)WALSH_ERR_TIMEOUT);
  if (warp == 1) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// 1 = ran, 0 = not applicable, < 0 = launch error
template <typename TU, typename TX>
static int launch_moe_experts_tc05(const void* u, int64_t ntok, const float* rw, const void* wgu, const void* wdown,
                                   const float* gammas, void* y, int fuse_post, const void* x, const float* hmix,
                                   void* xo, cudaStream_t s, int q0 = 0, int nq = 4) {
  using namespace moe_tc5;
  constexpr bool BF = std::is_same<TU, __nv_bfloat16>::value;
  CUtensorMap mu, mg, md;
  if (!make_tile_map(&mu, u, BF, ntok, C, 64, TOK) || !make_tile_map(&mg, wgu, BF, NPAIR * 256, 64, 64, 256) ||
      !make_tile_map(&md, wdown, BF, E * 32, HID, 64, 32))
    return 0;
  auto kern = moe_experts_tc05_kernel<TU, TX>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
    return launch_status();
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  const int64_t units = (ntok + TOK - 1) / TOK * nq;  // (tile, quarter of 4 experts)
  const unsigned grid = (unsigned)(units < sms ? units : sms);
  kern<<<grid, NTHREADS, SMEM, s>>>(mu, mg, md, ntok, rw, gammas, (TU*)y, fuse_post, (const TX*)x, hmix, (TX*)xo, q0,
                                    nq);
  const int st = launch_status();
  return st == WALSH_OK ? 1 : st;
}

int moe_tc05_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_moe_tc05_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_moe_tc05_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_moe_experts_tc_fwd(const void* u, int dtype, int64_t ntok, const float* weights,
                                                 const void* w_gu, const void* w_down, const float* gammas, void* y,
                                                 int fuse_post, const void* x, int x_dtype, const float* hmix,
                                                 void* x_out, void* stream) {
  if (int e = injected("moe_experts_tc_fwd")) return e;
  WALSH_CHECK_ARG(u && weights && w_gu && w_down && gammas);
  WALSH_CHECK_SHAPE(ntok >= 0 && ntok <= 2147483647LL);
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  if (fuse_post) {
    WALSH_CHECK_ARG(x && hmix && x_out);
    if (x_dtype != WALSH_BF16 && x_dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  } else {
    WALSH_CHECK_ARG(y);
  }
  if ((((uintptr_t)u) | ((uintptr_t)w_gu) | ((uintptr_t)w_down) | ((uintptr_t)x) | ((uintptr_t)x_out) |
       ((uintptr_t)y) | ((uintptr_t)hmix)) & 15u)
    return WALSH_ERR_ALIGN;
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  int r;
  const bool ubf = dtype == WALSH_BF16, xbf = !fuse_post || x_dtype == WALSH_BF16;
  if (ubf)
    r = xbf ? launch_moe_experts_tc05<__nv_bfloat16, __nv_bfloat16>(u, ntok, weights, w_gu, w_down, gammas, y,
                                                                     fuse_post, x, hmix, x_out, s)
            : launch_moe_experts_tc05<__nv_bfloat16, __half>(u, ntok, weights, w_gu, w_down, gammas, y, fuse_post,
                                                             x, hmix, x_out, s);
  else
    r = xbf ? launch_moe_experts_tc05<__half, __nv_bfloat16>(u, ntok, weights, w_gu, w_down, gammas, y, fuse_post,
                                                             x, hmix, x_out, s)
            : launch_moe_experts_tc05<__half, __half>(u, ntok, weights, w_gu, w_down, gammas, y, fuse_post, x, hmix,
                                                      x_out, s);
  return r == 1 ? WALSH_OK : (r == 0 ? WALSH_ERR_SHAPE : r);
}

extern "C" walsh_status walsh_moe_experts_tc_part_fwd(const void* u, int dtype, int64_t ntok, const float* weights,
                                                      const void* w_gu, const void* w_down, const float* gammas,
                                                      int first_expert, int n_experts, void* y, void* stream) {
  if (int e = injected("moe_experts_tc_part_fwd")) return e;
  WALSH_CHECK_ARG(u && weights && w_gu && w_down && gammas && y);
  WALSH_CHECK_SHAPE(ntok >= 0 && ntok <= 2147483647LL && first_expert >= 0 && n_experts >= 1 &&
                    first_expert + n_experts <= 16);
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  if ((((uintptr_t)u) | ((uintptr_t)w_gu) | ((uintptr_t)w_down) | ((uintptr_t)y)) & 15u) return WALSH_ERR_ALIGN;
  if (ntok == 0) return WALSH_OK;
  const int q0 = first_expert / 4, nq = (first_expert + n_experts + 3) / 4 - q0;
  cudaStream_t s = (cudaStream_t)stream;
  const int r = dtype == WALSH_BF16
                    ? launch_moe_experts_tc05<__nv_bfloat16, __nv_bfloat16>(u, ntok, weights, w_gu, w_down, gammas,
                                                                            y, 0, nullptr, nullptr, nullptr, s, q0, nq)
                    : launch_moe_experts_tc05<__half, __half>(u, ntok, weights, w_gu, w_down, gammas, y, 0, nullptr,
                                                              nullptr, nullptr, s, q0, nq);
  return r == 1 ? WALSH_OK : (r == 0 ? WALSH_ERR_SHAPE : r);
}

extern "C" walsh_status walsh_moe_fwd(const void* u, int dtype, int64_t ntok, int C, int top_k, const float* w1,
                                      const float* w2, const uint8_t* gate_2bit, const uint8_t* up_2bit,
                                      const uint8_t* down_2bit, const float* gammas, void* y, int fuse_post,
                                      const void* x, int x_dtype, const float* hmix, void* x_out,
                                      const float* weights_in, uint8_t* mask_out, float* probs_out,
                                      float* weights_out, const walsh_moe_tc_weights* tc,
                                      const walsh_moe_routing* routing, void* stream) {
  if (int e = injected("moe_fwd")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_DTYPE(x_dtype);
  const bool experts = gate_2bit || up_2bit || down_2bit;
  WALSH_CHECK_ARG(u);
  WALSH_CHECK_ARG(weights_in || (w1 && w2));                               // router needs its weights
  WALSH_CHECK_ARG(experts || !weights_in);                                // experts-only needs experts
  WALSH_CHECK_ARG(!experts || (gate_2bit && up_2bit && down_2bit && gammas));
  WALSH_CHECK_ARG(!experts || (fuse_post ? (x && hmix && x_out) : (y != nullptr)));
  WALSH_CHECK_SHAPE(ntok >= 0);
  WALSH_CHECK_SHAPE(top_k >= 1 && top_k <= MoeCfg<512>::MAXK && top_k <= C / 32);
  RouteRule rr;
  if (int e = make_route_rule(top_k, routing, &rr)) return e;
  WALSH_CHECK_ARG(!experts ||
                  ((((uintptr_t)gate_2bit | (uintptr_t)up_2bit) & 7u) == 0 && ((uintptr_t)down_2bit & 15u) == 0));
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype != WALSH_F32 && C == 512 && tc && tc->w1 && tc->w2 && !weights_in &&
      (!experts || (tc->gate && tc->up && tc->down)) &&
      (!fuse_post || x_dtype == WALSH_BF16 || x_dtype == WALSH_F16) &&
      ((((uintptr_t)u) | ((uintptr_t)tc->w1) | ((uintptr_t)tc->w2) | ((uintptr_t)tc->gate) |
        ((uintptr_t)tc->up) | ((uintptr_t)tc->down) | ((uintptr_t)y) | ((uintptr_t)x) | ((uintptr_t)x_out) |
        ((uintptr_t)hmix)) & 15u) == 0) {
    const bool xh = fuse_post && x_dtype == WALSH_F16;  // stream type of the fused epilogue
    if (dtype == WALSH_F16)
      return xh ? launch_moe_mma<__half, __half>(u, ntok, rr, tc, experts, gammas, y, fuse_post, x, hmix, x_out,
                                                 mask_out, probs_out, weights_out, s)
                : launch_moe_mma<__half, __nv_bfloat16>(u, ntok, rr, tc, experts, gammas, y, fuse_post, x, hmix,
                                                        x_out, mask_out, probs_out, weights_out, s);
    return xh ? launch_moe_mma<__nv_bfloat16, __half>(u, ntok, rr, tc, experts, gammas, y, fuse_post, x, hmix,
                                                      x_out, mask_out, probs_out, weights_out, s)
              : launch_moe_mma<__nv_bfloat16, __nv_bfloat16>(u, ntok, rr, tc, experts, gammas, y, fuse_post, x,
                                                             hmix, x_out, mask_out, probs_out, weights_out, s);
  }
  if (C != 512 && C != 2048) return WALSH_ERR_SHAPE;
  return WALSH_DISPATCH_DTYPE(dtype, TU, WALSH_DISPATCH_DTYPE(x_dtype, TX,
      C == 512 ? launch_moe<TU, TX, 512>(u, ntok, rr, w1, w2, gate_2bit, up_2bit, down_2bit, gammas, y, fuse_post,
                                         x, hmix, x_out, weights_in, mask_out, probs_out, weights_out, s)
               : launch_moe<TU, TX, 2048>(u, ntok, rr, w1, w2, gate_2bit, up_2bit, down_2bit, gammas, y,
                                          fuse_post, x, hmix, x_out, weights_in, mask_out, probs_out, weights_out,
                                          s)));
}

extern "C" walsh_status walsh_moe_hidden_fwd(const void* u, const void* hpre, int dtype, int64_t ntok, int C,
                                             int top_k, const float* w2, const uint8_t* gate_2bit,
                                             const uint8_t* up_2bit, const uint8_t* down_2bit, const float* gammas,
                                             void* y, int fuse_post, const void* x, int x_dtype, const float* hmix,
                                             void* x_out, uint8_t* mask_out, float* probs_out, float* weights_out,
                                             const walsh_moe_routing* routing, void* stream) {
  if (int e = injected("moe_hidden_fwd")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_DTYPE(x_dtype);
  WALSH_CHECK_ARG(u && hpre && w2 && gate_2bit && up_2bit && down_2bit && gammas);
  WALSH_CHECK_ARG(fuse_post ? (x && hmix && x_out) : (y != nullptr));
  WALSH_CHECK_SHAPE(ntok >= 0 && (C == 512 || C == 2048));
  WALSH_CHECK_SHAPE(top_k >= 1 && top_k <= 8 && top_k <= C / 32);
  RouteRule rr;
  if (int e = make_route_rule(top_k, routing, &rr)) return e;
  WALSH_CHECK_ARG(((((uintptr_t)gate_2bit | (uintptr_t)up_2bit) & 7u) == 0) && (((uintptr_t)down_2bit & 15u) == 0) &&
                  (((uintptr_t)w2 & 15u) == 0) && (!fuse_post || ((((uintptr_t)x) | ((uintptr_t)x_out)) & 15u) == 0));
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  return WALSH_DISPATCH_DTYPE(dtype, TU, WALSH_DISPATCH_DTYPE(x_dtype, TX,
      C == 512 ? launch_moe_token<TU, TX, 512>(u, hpre, ntok, rr, w2, gate_2bit, up_2bit, down_2bit, gammas, y,
                                               fuse_post, x, hmix, x_out, mask_out, probs_out, weights_out, s)
               : launch_moe_token<TU, TX, 2048>(u, hpre, ntok, rr, w2, gate_2bit, up_2bit, down_2bit, gammas,
                                                y, fuse_post, x, hmix, x_out, mask_out, probs_out, weights_out, s)));
}
