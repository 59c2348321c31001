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

template <typename T, int C>
__global__ void __launch_bounds__(256)
moe_kernel(const T* __restrict__ u, int64_t ntok, int top_k, const float* __restrict__ w1t,
           const float* __restrict__ w2, const uint8_t* __restrict__ gp, const uint8_t* __restrict__ upp,
           const uint8_t* __restrict__ dp, const float* __restrict__ gammas, T* __restrict__ y, int fuse_post,
           const T* x, const float* __restrict__ hmix, T* xo, const float* __restrict__ weights_in,
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
#pragma unroll 4
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
#pragma unroll 8
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
    for (int k = 0; k < top_k; ++k) {
      int best = -1;
      float bv = -1.f;
      for (int e = 0; e < E; ++e)
        if (!((chosen >> e) & 1ull) && l[e] > bv) { bv = l[e]; best = e; }
      if (best < 0) {  // non-finite scores: take the lowest unchosen expert so indices stay in range
        for (int e = E - 1; e >= 0; --e)
          if (!((chosen >> e) & 1ull)) best = e;
        bv = 0.f;
      }
      chosen |= 1ull << best;
      sel[tid * E + k] = best;
      selw[tid * E + k] = bv;
    }
    nsel[tid] = top_k;
    // renormalise in ascending expert order, as (probs * mask).sum(-1) does
    for (int e = 0; e < E; ++e)
      if ((chosen >> e) & 1ull) wsum += l[e];
    wsum = fmaxf(wsum, 1e-8f);
    for (int k = 0; k < top_k; ++k) selw[tid * E + k] = __fdiv_rn(selw[tid * E + k], wsum);
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
  const int slots = weights_in ? E : top_k;
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
      xo[base + (size_t)r * C] = from_f<T>(v);
    }
  }
}

template <typename T, int C>
static int launch_moe(const void* u, int64_t ntok, int top_k, const float* w1t, const float* w2, const uint8_t* gp,
                      const uint8_t* upp, const uint8_t* dp, const float* gammas, void* y, int fuse_post,
                      const void* x, const float* hmix, void* xo, const float* weights_in, uint8_t* mask_out,
                      float* probs_out, float* weights_out, cudaStream_t s) {
  using M = MoeCfg<C>;
  const size_t smem = (2 * M::TM * C + M::TM * M::HID + M::TM * M::E + 8 * kExpertHidden) * sizeof(float) +
                      M::TM * M::E * (sizeof(int) + sizeof(float)) + M::TM * sizeof(int);
  auto kern = moe_kernel<T, C>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (ntok + M::TM - 1) / M::TM;
  kern<<<(unsigned)grid, 256, smem, s>>>((const T*)u, ntok, top_k, w1t, w2, gp, upp, dp, gammas, (T*)y, fuse_post,
                                         (const T*)x, hmix, (T*)xo, weights_in, mask_out, probs_out, weights_out);
  return launch_status();
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_moe_fwd(const void* u, int dtype, int64_t ntok, int C, int top_k, const float* w1,
                                      const float* w2, const uint8_t* gate_2bit, const uint8_t* up_2bit,
                                      const uint8_t* down_2bit, const float* gammas, void* y, int fuse_post,
                                      const void* x, const float* hmix, void* x_out, const float* weights_in,
                                      uint8_t* mask_out, float* probs_out, float* weights_out, void* stream) {
  if (int e = injected("moe_fwd")) return e;
  WALSH_CHECK_DTYPE(dtype);
  const bool experts = gate_2bit || up_2bit || down_2bit;
  WALSH_CHECK_ARG(u);
  WALSH_CHECK_ARG(weights_in || (w1 && w2));                               // router needs its weights
  WALSH_CHECK_ARG(experts || !weights_in);                                // experts-only needs experts
  WALSH_CHECK_ARG(!experts || (gate_2bit && up_2bit && down_2bit && gammas));
  WALSH_CHECK_ARG(!experts || (fuse_post ? (x && hmix && x_out) : (y != nullptr)));
  WALSH_CHECK_SHAPE(ntok >= 0);
  WALSH_CHECK_SHAPE(top_k >= 1 && top_k <= MoeCfg<512>::MAXK && top_k <= C / 32);
  WALSH_CHECK_ARG(!experts ||
                  ((((uintptr_t)gate_2bit | (uintptr_t)up_2bit) & 7u) == 0 && ((uintptr_t)down_2bit & 15u) == 0));
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
#define WALSH_MOE_CASE(CC)                                                                                    \
  if (C == CC)                                                                                               \
    return dtype == WALSH_F32                                                                                \
               ? launch_moe<float, CC>(u, ntok, top_k, w1, w2, gate_2bit, up_2bit, down_2bit, gammas, y,    \
                                       fuse_post, x, hmix, x_out, weights_in, mask_out, probs_out,          \
                                       weights_out, s)                                                      \
               : launch_moe<__nv_bfloat16, CC>(u, ntok, top_k, w1, w2, gate_2bit, up_2bit, down_2bit,      \
                                               gammas, y, fuse_post, x, hmix, x_out, weights_in, mask_out,  \
                                               probs_out, weights_out, s);
  WALSH_MOE_CASE(512)
  WALSH_MOE_CASE(2048)
#undef WALSH_MOE_CASE
  return WALSH_ERR_SHAPE;
}
