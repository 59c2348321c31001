// mHC residual-stream kernels (n_streams = 4).
//
// walsh_mhc_map fuses, per token, the three ResidualStreamMapping.forward
// calls (src/model/mhc.py:283-318) -- which each recompute the same weightless
// RMSNorm of x_flat -- into one pass over x: one sum of squares, one
// [24 x 4C] projection, then sigmoid / 2*sigmoid / Sinkhorn-20 in registers,
// followed by the pre-mix H_pre @ x (src/model/mhc.py:364) and the block's
// attention_norm / ffn_norm RMSNorm (src/model/mhc.py:514-523).
#include <stdlib.h>
#include <type_traits>

#include "common.cuh"
#include "mma.cuh"
#include "tc05.cuh"
#include "tma_host.cuh"

namespace walsh {

// Sinkhorn-Knopp on a 4x4 matrix held in registers (src/model/mhc.py:214-229):
// exp, then `iters` x (column, row) normalisation.  Each normalisation takes one
// hardware reciprocal of (sum + eps) (rcp.approx, within about one ulp; the
// sums are at least eps, so never subnormal) and four multiplies: within two
// ulps of the reference's four divisions per line.  A correctly rounded
// reciprocal takes several instructions per call, and the normalisations are
// most of the per-token activation work.
__device__ __forceinline__ float rcp_fast(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void sinkhorn4(float* M, int iters, float eps) {
#pragma unroll
  for (int i = 0; i < 16; ++i) M[i] = expf(M[i]);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float inv = rcp_fast((((M[c] + M[4 + c]) + M[8 + c]) + M[12 + c]) + eps);
#pragma unroll
      for (int r = 0; r < 4; ++r) M[4 * r + c] *= inv;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float inv = rcp_fast((((M[4 * r] + M[4 * r + 1]) + M[4 * r + 2]) + M[4 * r + 3]) + eps);
#pragma unroll
      for (int c = 0; c < 4; ++c) M[4 * r + c] *= inv;
    }
  }
}

// Turns the 24 raw projections d (already multiplied by the RMS factor) into
// {H_pre[4], H_post[4], H_res[16]}.
__device__ __forceinline__ void map_activations(const float* d, const float* __restrict__ mp, float* hm) {
  const float a_pre = __ldg(mp + 0), a_post = __ldg(mp + 1), a_res = __ldg(mp + 2);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    hm[j] = 1.0f / (1.0f + expf(-(a_pre * d[j] + __ldg(mp + 4 + j))));
    hm[4 + j] = 2.0f * (1.0f / (1.0f + expf(-(a_post * d[4 + j] + __ldg(mp + 8 + j)))));
  }
  float M[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) M[i] = a_res * d[8 + i] + __ldg(mp + 12 + i);
  sinkhorn4(M, 20, 1e-8f);
#pragma unroll
  for (int i = 0; i < 16; ++i) hm[8 + i] = M[i];
}

// CTA = 8 warps x TPW tokens.  phi is staged through shared memory in chunks
// of KC columns so that each phi value read serves TPW tokens.
template <typename T, typename TU, int TPW>
__global__ void __launch_bounds__(256)
mhc_map_kernel(const T* __restrict__ x, int64_t ntok, int C, const float* __restrict__ phi,
               const float* __restrict__ mp, float map_eps, const float* __restrict__ norm_w, float norm_eps,
               TU* __restrict__ u, float* __restrict__ hmix) {
  constexpr int KC = 128;
  extern __shared__ float4 smem4[];
  float* phis = reinterpret_cast<float*>(smem4);      // [24][KC]
  float* hs = phis + kMapRows * KC;                    // [8][TPW][24]
  float* us = hs + 8 * TPW * kMapRows;                 // [8][C]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = 4 * C;
  const int64_t tok0 = ((int64_t)blockIdx.x * 8 + warp) * TPW;
  float acc[TPW][kMapRows];
  float ss[TPW];
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
    ss[t] = 0.f;
#pragma unroll
    for (int r = 0; r < kMapRows; ++r) acc[t][r] = 0.f;
  }
  for (int k0 = 0; k0 < D; k0 += KC) {
    __syncthreads();
    for (int i = threadIdx.x; i < kMapRows * KC; i += 256) {
      const int r = i / KC, kk = i - r * KC;
      phis[i] = __ldg(phi + (size_t)r * D + k0 + kk);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < KC / 32; ++j) {
      const int kk = lane + 32 * j;
      float xv[TPW];
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        xv[t] = (tok0 + t < ntok) ? to_f(x[(tok0 + t) * D + k0 + kk]) : 0.f;
        ss[t] = fmaf(xv[t], xv[t], ss[t]);
      }
#pragma unroll
      for (int r = 0; r < kMapRows; ++r) {
        const float w = phis[r * KC + kk];
#pragma unroll
        for (int t = 0; t < TPW; ++t) acc[t][r] = fmaf(w, xv[t], acc[t][r]);
      }
    }
  }
  // reduce across the warp; lane t < TPW keeps token t's values
  float mine[kMapRows];
  float myss = 0.f;
#pragma unroll
  for (int r = 0; r < kMapRows; ++r) mine[r] = 0.f;
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
    const float s = warp_sum(ss[t]);
    if (lane == t) myss = s;
#pragma unroll
    for (int r = 0; r < kMapRows; ++r) {
      const float v = warp_sum(acc[t][r]);
      if (lane == t) mine[r] = v;
    }
  }
  float* hw = hs + warp * TPW * kMapRows;
  if (lane < TPW) {
    const float rms = rsqrtf(myss / (float)D + map_eps);
    float d[kMapRows], hm[kMapRows];
#pragma unroll
    for (int r = 0; r < kMapRows; ++r) d[r] = mine[r] * rms;
    map_activations(d, mp, hm);
#pragma unroll
    for (int r = 0; r < kMapRows; ++r) hw[lane * kMapRows + r] = hm[r];
  }
  __syncwarp();
  float* uw = us + warp * C;
#pragma unroll 1
  for (int t = 0; t < TPW; ++t) {
    const int64_t tok = tok0 + t;
    if (tok >= ntok) break;
    if (lane < kMapRows) hmix[tok * kMapRows + lane] = hw[t * kMapRows + lane];
    const float h0 = hw[t * kMapRows + 0], h1 = hw[t * kMapRows + 1];
    const float h2 = hw[t * kMapRows + 2], h3 = hw[t * kMapRows + 3];
    const T* xt = x + tok * D;
    float s2 = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = ((h0 * to_f(xt[c]) + h1 * to_f(xt[C + c])) + h2 * to_f(xt[2 * C + c])) + h3 * to_f(xt[3 * C + c]);
      uw[c] = v;
      s2 = fmaf(v, v, s2);
    }
    s2 = warp_sum(s2);
    const float rn = norm_w ? rsqrtf(s2 / (float)C + norm_eps) : 1.0f;
    TU* ut = u + tok * C;
    for (int c = lane; c < C; c += 32) {
      const float v = uw[c] * rn;
      ut[c] = from_f<TU>(norm_w ? v * __ldg(norm_w + c) : v);
    }
    __syncwarp();
  }
}

// bf16 variant on the tensor cores: CTA = 8 warps x 16 tokens.  The CTA
// streams its 128 tokens' 4C values and the matching 128-column chunk of phi
// (bf16 copy, [24, 4C]) through double-buffered shared memory with cp.async;
// each warp runs m16n8k16 MMAs for its 16 tokens with both operands from
// shared memory (ldmatrix) and takes the sum of squares from the same A
// fragments.  Then lanes 0..15 finish one token each (RMS factor, sigmoid /
// Sinkhorn) and the warp does the pre-mix + RMSNorm per token.
namespace map_tc {
constexpr int NW = 8, TOK = NW * 16, KC = 128, LDX = KC + 8;
template <int C>
constexpr size_t smem_bytes() {
  return (size_t)2 * (TOK + kMapRows) * LDX * sizeof(__nv_bfloat16) + (size_t)NW * 16 * (kMapRows + 1) * sizeof(float) +
         (size_t)NW * 16 * sizeof(float);
}
}  // namespace map_tc

template <int C, typename TU, typename TX>
__global__ void __launch_bounds__(256)
mhc_map_mma_kernel(const TX* __restrict__ x, int64_t ntok, const TX* __restrict__ phib,
                   const float* __restrict__ mp, float map_eps, const float* __restrict__ norm_w, float norm_eps,
                   TU* __restrict__ u, float* __restrict__ hmix) {
  using namespace map_tc;
  constexpr int D = 4 * C, NCH = D / KC;
  extern __shared__ float4 smem4[];
  TX* xs = reinterpret_cast<TX*>(smem4);   // [2][TOK][LDX]
  TX* ps = xs + 2 * TOK * LDX;                          // [2][24][LDX]
  float (*ds)[16][kMapRows + 1] = reinterpret_cast<float (*)[16][kMapRows + 1]>(ps + 2 * kMapRows * LDX);
  float (*sss)[16] = reinterpret_cast<float (*)[16]>(reinterpret_cast<float*>(ds) + NW * 16 * (kMapRows + 1));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int64_t cta0 = (int64_t)blockIdx.x * TOK;
  const int64_t tok0 = cta0 + warp * 16;

  auto load_chunk = [&](int ch, int buf) {
    TX* xd = xs + buf * TOK * LDX;
    for (int i = tid; i < TOK * (KC / 8); i += 256) {
      const int r = i / (KC / 8), c = i - r * (KC / 8);
      const bool in = cta0 + r < ntok;
      cp_async16(xd + r * LDX + c * 8, x + (in ? (cta0 + r) * D : 0) + ch * KC + c * 8, in ? 16 : 0);
    }
    TX* pd = ps + buf * kMapRows * LDX;
    for (int i = tid; i < kMapRows * (KC / 8); i += 256) {
      const int r = i / (KC / 8), c = i - r * (KC / 8);
      cp_async16(pd + r * LDX + c * 8, phib + (size_t)r * D + ch * KC + c * 8, 16);
    }
  };
  float acc[3][4];
#pragma unroll
  for (int n = 0; n < 3; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float ss_lo = 0.f, ss_hi = 0.f;
  load_chunk(0, 0);
  cp_async_commit();
  for (int ch = 0; ch < NCH; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < NCH) load_chunk(ch + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const TX* xw = xs + buf * TOK * LDX + warp * 16 * LDX;
    const TX* pw = ps + buf * kMapRows * LDX;
#pragma unroll
    for (int ks = 0; ks < KC / 16; ++ks) {
      uint32_t a[4], b01[4], b2[2];
      ldsm_x4(a, xw + (lane & 15) * LDX + ks * 16 + (lane >> 4) * 8);
      ldsm_x4(b01, pw + ((lane & 7) + ((lane >> 4) << 3)) * LDX + ks * 16 + ((lane >> 3) & 1) * 8);
      ldsm_x2(b2[0], b2[1], pw + (16 + (lane & 7)) * LDX + ks * 16 + ((lane >> 3) & 1) * 8);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float2 v = unpack2<TX>(a[r]);
        if (r & 1) ss_hi = fmaf(v.x, v.x, fmaf(v.y, v.y, ss_hi));
        else ss_lo = fmaf(v.x, v.x, fmaf(v.y, v.y, ss_lo));
      }
      mma16<TX>(acc[0], a, b01[0], b01[1]);
      mma16<TX>(acc[1], a, b01[2], b01[3]);
      mma16<TX>(acc[2], a, b2[0], b2[1]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    ss_lo += __shfl_xor_sync(0xffffffffu, ss_lo, off);
    ss_hi += __shfl_xor_sync(0xffffffffu, ss_hi, off);
  }
#pragma unroll
  for (int n = 0; n < 3; ++n) {
    ds[warp][g][8 * n + 2 * t4] = acc[n][0];
    ds[warp][g][8 * n + 2 * t4 + 1] = acc[n][1];
    ds[warp][g + 8][8 * n + 2 * t4] = acc[n][2];
    ds[warp][g + 8][8 * n + 2 * t4 + 1] = acc[n][3];
  }
  if (t4 == 0) {
    sss[warp][g] = ss_lo;
    sss[warp][g + 8] = ss_hi;
  }
  __syncwarp();
  if (lane < 16) {
    const float rms = rsqrtf(sss[warp][lane] / (float)D + map_eps);
    float d[kMapRows], hm[kMapRows];
#pragma unroll
    for (int r = 0; r < kMapRows; ++r) d[r] = ds[warp][lane][r] * rms;
    map_activations(d, mp, hm);
#pragma unroll
    for (int r = 0; r < kMapRows; ++r) ds[warp][lane][r] = hm[r];
    if (tok0 + lane < ntok) {
#pragma unroll
      for (int r = 0; r < kMapRows; ++r) hmix[(tok0 + lane) * kMapRows + r] = hm[r];
    }
  }
  __syncwarp();
  // pre-mix u = sum_j H_pre[j] x_j and the block RMSNorm, 8 columns per lane per step;
  // for C = 512 token t + 1's stream rows are loaded before token t is computed
  constexpr int VPL = C / 256;  // uint4 chunks per lane
  constexpr bool PREFETCH = VPL <= 2;  // two tokens' rows fit in registers
  uint4 xr[VPL][4];
  auto load_tok = [&](int64_t tok, uint4 (&dst)[VPL][4]) {
    const TX* xt = x + tok * D;
#pragma unroll
    for (int v = 0; v < VPL; ++v)
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[v][j] = __ldg(reinterpret_cast<const uint4*>(xt + j * C + (lane + 32 * v) * 8));
  };
  if (PREFETCH && tok0 < ntok) load_tok(tok0, xr);
  for (int t = 0; t < 16; ++t) {
    const int64_t tok = tok0 + t;
    if (tok >= ntok) break;
    uint4 xn[VPL][4];
    if (PREFETCH) {
      if (t + 1 < 16 && tok + 1 < ntok) load_tok(tok + 1, xn);
    } else {
      load_tok(tok, xr);
    }
    const float h0 = ds[warp][t][0], h1 = ds[warp][t][1], h2 = ds[warp][t][2], h3 = ds[warp][t][3];
    float uv[VPL][8];
    float s2 = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      float f0[8], f1[8], f2[8], f3[8];
      unpack8(xr[v][0], f0, (const TX*)nullptr);
      unpack8(xr[v][1], f1, (const TX*)nullptr);
      unpack8(xr[v][2], f2, (const TX*)nullptr);
      unpack8(xr[v][3], f3, (const TX*)nullptr);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uv[v][e] = ((h0 * f0[e] + h1 * f1[e]) + h2 * f2[e]) + h3 * f3[e];
        s2 = fmaf(uv[v][e], uv[v][e], s2);
      }
    }
    if (PREFETCH) {
#pragma unroll
      for (int v = 0; v < VPL; ++v)
#pragma unroll
        for (int j = 0; j < 4; ++j) xr[v][j] = xn[v][j];
    }
    s2 = warp_sum(s2);
    const float rn = norm_w ? rsqrtf(s2 / (float)C + norm_eps) : 1.0f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (lane + 32 * v) * 8;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = uv[v][e] * rn * (norm_w ? __ldg(norm_w + c + e) : 1.f);
      store8(u + tok * C + c, o);
    }
  }
}

// ---------------------------------------------------------------------------
// Single-pass site prologue for C = 512 (16-bit x): 16 tokens per CTA, their
// whole stream rows (16 x 2048 x 2 B = 64 KB) loaded once by TMA into shared
// memory (32 boxes of 64 columns x 16 rows, 128-byte swizzle), then
//   1. the 8 warps split the 2048 columns (256 each): sum of squares and the
//      24 projections on the tensor cores, A = x from shared memory through
//      ldmatrix, B = phi pre-arranged in MMA-fragment order and read from L2;
//   2. one thread per token adds the 8 partials, applies the RMS scale,
//      sigmoid / 2 sigmoid / Sinkhorn and writes hmix;
//   3. the pre-mix u = sum_j H_pre[j] x_j and the block RMSNorm from shared
//      memory, two tokens per warp.
// x is read from HBM once (the two-pass kernel reads it twice).
// ---------------------------------------------------------------------------
// TOKN tokens per CTA: 16 (C = 512, 64 KB of x) or 8 (C = 2048: 128 KB; and
// C = 512 at small token counts, for twice the CTAs).  With 8 the MMA's rows
// 8..15 read the next box (the last box: the reduction scratch after it) and
// are discarded.
template <int C, int TOKN>
struct MapTma {
  static constexpr int TOK = TOKN, NW = 8, D = 4 * C, BOXC = 64, NBOX = D / BOXC;
  static constexpr int BOX_BYTES = TOK * BOXC * 2;
  static constexpr int X_BYTES = NBOX * BOX_BYTES;
  static constexpr int RED_FLOATS = NW * 16 * (kMapRows + 1);
  static constexpr int SMEM = X_BYTES + RED_FLOATS * 4 + TOK * kMapRows * 4 + 1024 + 64;
  // shared-memory byte offset of x[row][col] in the swizzled box layout
  __device__ static __forceinline__ uint32_t off(int row, int col) {
    const int b = col >> 6, ch = (col & 63) >> 3;
    return (uint32_t)(b * BOX_BYTES + row * 128 + ((ch ^ (row & 7)) << 4) + ((col & 7) << 1));
  }
};

__device__ int g_map_tma_error;

template <int C, typename TX, typename TU, int TOKN>
__global__ void __launch_bounds__(256)
mhc_map_tma_kernel(const __grid_constant__ CUtensorMap tmx, int64_t ntok, const uint2* __restrict__ phif,
                   const float* __restrict__ mp, float map_eps, const float* __restrict__ norm_w, float norm_eps,
                   TU* __restrict__ u, float* __restrict__ hmix) {
  using G = MapTma<C, TOKN>;
  constexpr int TOK = G::TOK, NW = G::NW, D = G::D, BOXC = G::BOXC, NBOX = G::NBOX, BOX_BYTES = G::BOX_BYTES,
                X_BYTES = G::X_BYTES, RED_FLOATS = G::RED_FLOATS;
  constexpr int KS = D / 16 / NW;  // k-steps per warp
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* xs = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* red = reinterpret_cast<float*>(xs + X_BYTES);  // [NW][16][25]
  float* hc = red + RED_FLOATS;                         // [TOK][24]
  uint64_t* bar = reinterpret_cast<uint64_t*>(hc + TOK * kMapRows);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int64_t tok0 = (int64_t)blockIdx.x * TOK;
  if (tid == 0) {
    tc05::mbar_init(bar, 1);
    tc05::fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    tc05::prefetch_tensormap(&tmx);
    tc05::mbar_arrive_expect_tx(bar, X_BYTES);
    for (int b = 0; b < NBOX; ++b) tc05::tma_load_2d(xs + b * BOX_BYTES, &tmx, bar, b * BOXC, (int)tok0);
  }
  // 1. partial projections over this warp's columns; the first 16 k-steps'
  // phi fragments are loaded while the TMA copies are in flight
  constexpr int KB = KS < 16 ? KS : 16;  // k-steps per fragment batch
  uint2 fr[KB][3];
  auto load_frags = [&](int kb) {
#pragma unroll
    for (int j = 0; j < KB; ++j) {
      const uint2* fp = phif + ((size_t)(kb + j) * 32 + lane) * 3;
      fr[j][0] = __ldg(fp);
      fr[j][1] = __ldg(fp + 1);
      fr[j][2] = __ldg(fp + 2);
    }
  };
  load_frags(warp * KS);
  if (!tc05::mbar_wait(bar, 0)) {
    if (tid == 0) atomicExch(&g_map_tma_error, (int)WALSH_ERR_TIMEOUT);
    return;
  }
  float acc[3][4];
#pragma unroll
  for (int n = 0; n < 3; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float ss_lo = 0.f, ss_hi = 0.f;
  const uint32_t xbase = tc05::smem_u32(xs);
#pragma unroll 1
  for (int kb8 = warp * KS; kb8 < warp * KS + KS; kb8 += KB) {
    if (kb8 != warp * KS) load_frags(kb8);
#pragma unroll
    for (int j = 0; j < KB; ++j) {
      const int ks = kb8 + j;
      const int r = lane & 15, col = ks * 16 + (lane >> 4) * 8;
      uint32_t a[4];
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                   : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                   : "r"(xbase + G::off(r, col)));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = unpack2<TX>(a[q]);
        if (q & 1) ss_hi = fmaf(v.x, v.x, fmaf(v.y, v.y, ss_hi));
        else ss_lo = fmaf(v.x, v.x, fmaf(v.y, v.y, ss_lo));
      }
      mma16<TX>(acc[0], a, fr[j][0].x, fr[j][0].y);
      mma16<TX>(acc[1], a, fr[j][1].x, fr[j][1].y);
      mma16<TX>(acc[2], a, fr[j][2].x, fr[j][2].y);
    }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    ss_lo += __shfl_xor_sync(0xffffffffu, ss_lo, off);
    ss_hi += __shfl_xor_sync(0xffffffffu, ss_hi, off);
  }
  float* rw = red + warp * 16 * (kMapRows + 1);
#pragma unroll
  for (int n = 0; n < 3; ++n) {
    rw[g * (kMapRows + 1) + 8 * n + 2 * t4] = acc[n][0];
    rw[g * (kMapRows + 1) + 8 * n + 2 * t4 + 1] = acc[n][1];
    rw[(g + 8) * (kMapRows + 1) + 8 * n + 2 * t4] = acc[n][2];
    rw[(g + 8) * (kMapRows + 1) + 8 * n + 2 * t4 + 1] = acc[n][3];
  }
  if (t4 == 0) {
    rw[g * (kMapRows + 1) + kMapRows] = ss_lo;
    rw[(g + 8) * (kMapRows + 1) + kMapRows] = ss_hi;
  }
  __syncthreads();
  // 2a. per-token sums of the 8 warps' partials (warp order fixed): ds[t][v], v < 25
  float* ds = red;  // reused in place: column v of warp 0's rows
  {
    float tmp[2] = {0.f, 0.f};
    const int t = tid >> 4, e = tid & 15;
    if (t < TOK) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = e + 16 * k;
        if (v <= kMapRows)
          for (int w = 0; w < NW; ++w) tmp[k] += red[(w * 16 + t) * (kMapRows + 1) + v];
      }
    }
    __syncthreads();
    if (t < TOK) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = e + 16 * k;
        if (v <= kMapRows) ds[t * (kMapRows + 1) + v] = tmp[k];
      }
    }
  }
  __syncthreads();
  // 2b. activations, 16 threads per token (one per H_res entry): thread e of token t
  //     holds M[e] (row e / 4, column e % 4) and gathers columns and rows by shuffles,
  //     adding in the same order as the single-thread sinkhorn4
  if (tid < TOK * 16) {
    const int t = tid >> 4, e = tid & 15, base = lane & 16, r = e >> 2, c = e & 3;
    const float* dt = ds + t * (kMapRows + 1);
    const float rms = rsqrtf(dt[kMapRows] / (float)D + map_eps);
    const float a_pre = __ldg(mp + 0), a_post = __ldg(mp + 1), a_res = __ldg(mp + 2);
    const int64_t tok = tok0 + t;
    if (e < 4) {
      const float hp = 1.0f / (1.0f + expf(-(a_pre * (dt[e] * rms) + __ldg(mp + 4 + e))));
      hc[t * kMapRows + e] = hp;
      if (tok < ntok) hmix[tok * kMapRows + e] = hp;
    } else if (e < 8) {
      const float ho = 2.0f * (1.0f / (1.0f + expf(-(a_post * (dt[e] * rms) + __ldg(mp + 8 + (e - 4))))));
      if (tok < ntok) hmix[tok * kMapRows + e] = ho;
    }
    float M = expf(a_res * (dt[8 + e] * rms) + __ldg(mp + 12 + e));
    for (int it = 0; it < 20; ++it) {
      const float c0 = __shfl_sync(0xffffffffu, M, base + c), c1 = __shfl_sync(0xffffffffu, M, base + 4 + c),
                  c2 = __shfl_sync(0xffffffffu, M, base + 8 + c), c3 = __shfl_sync(0xffffffffu, M, base + 12 + c);
      M *= rcp_fast((((c0 + c1) + c2) + c3) + 1e-8f);
      const float r0 = __shfl_sync(0xffffffffu, M, base + 4 * r), r1 = __shfl_sync(0xffffffffu, M, base + 4 * r + 1),
                  r2 = __shfl_sync(0xffffffffu, M, base + 4 * r + 2),
                  r3 = __shfl_sync(0xffffffffu, M, base + 4 * r + 3);
      M *= rcp_fast((((r0 + r1) + r2) + r3) + 1e-8f);
    }
    if (tok < ntok) hmix[tok * kMapRows + 8 + e] = M;
  }
  __syncthreads();
  // 3. pre-mix and RMSNorm: TOK / NW tokens per warp; lane covers C / 32 columns
  constexpr int VPL = C / 256;
#pragma unroll 1
  for (int tt = 0; tt < TOK / NW; ++tt) {
    const int t = warp * (TOK / NW) + tt;
    const int64_t tok = tok0 + t;
    if (tok >= ntok) break;
    const float h0 = hc[t * kMapRows], h1 = hc[t * kMapRows + 1], h2 = hc[t * kMapRows + 2],
                h3 = hc[t * kMapRows + 3];
    float uv[VPL][8];
    float s2 = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (lane + 32 * v) * 8;
      float f[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 q = *reinterpret_cast<const uint4*>(xs + G::off(t, j * C + c));
        unpack8(q, f[j], (const TX*)nullptr);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uv[v][e] = ((h0 * f[0][e] + h1 * f[1][e]) + h2 * f[2][e]) + h3 * f[3][e];
        s2 = fmaf(uv[v][e], uv[v][e], s2);
      }
    }
    s2 = warp_sum(s2);
    const float rn = norm_w ? rsqrtf(s2 / (float)C + norm_eps) : 1.0f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (lane + 32 * v) * 8;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = uv[v][e] * rn * (norm_w ? __ldg(norm_w + c + e) : 1.f);
      store8(u + tok * C + c, o);
    }
  }
}

// ---------------------------------------------------------------------------
// Prefill-sized mapping (C = 512, 16-bit x), x read from HBM once.  One CTA
// per SM walks 16-token tiles (a tile's stream rows are one contiguous 64 KB
// block).  The rows come through a ring of STAGES shared-memory buffers, one
// bulk copy (cp.async.bulk, completing on the stage's mbarrier) per 4 KB
// token row into rows padded by 16 bytes so that ldmatrix's eight rows fall
// in distinct banks; thread 0 refills a stage with the tile STAGES ahead as
// soon as the stage is released, so the next tiles' loads run while the
// current one is computed.  Sixteen main warps do, per tile:
//   1. projections and sum of squares on the tensor cores from shared memory,
//      each warp a 128-column slice of the 16 tokens (the slice's phi
//      fragments stay in registers for all tiles), partials to shared memory;
//   2. warp w then adds token w's 16 partials (lane v: index v, warp order),
//      takes the RMS factor, H_pre / H_post, the pre-exponential H_res logits
//      (posted to shared memory for the Sinkhorn warp) and the pre-mix
//      u = sum_j H_pre[j] x_j with the block RMSNorm, reading the stream rows
//      from the ring buffer, which is then refilled with the tile STAGES ahead.
// A 17th warp runs the 16 tokens' Sinkhorn of each tile (one token per lane,
// in registers) while the main warps go on with the next tile; two named
// barriers hand the logits over (full: main warps arrive, Sinkhorn warp
// waits; empty: the reverse).  Every mbarrier wait is bounded: if one runs
// out, the main warps record WALSH_ERR_TIMEOUT (walsh_map_error), release
// the Sinkhorn warp through the same barriers with an abort flag, wait
// (bounded) for the copies they have in flight and return.
// Measured at 65 536 tokens: with the Sinkhorn on warp 0, 182 us (45 of them
// Sinkhorn); the Sinkhorn warp with 16-byte cp.async loads, 140 us; a TMA form
// of the ring (32 boxes of 64 columns x 16 rows per tile), 190 us; the
// two-pass kernel 142 us.
// ---------------------------------------------------------------------------
namespace map_pipe {
constexpr int STAGES = 2, TOK = 16, NW = 16, THREADS = (NW + 1) * 32, C = 512, D = 4 * C;
constexpr int ROWB = D * 2 + 16;             // bytes per token row in shared memory (padded)
constexpr int STAGE_BYTES = TOK * ROWB;
constexpr int RS = kMapRows + 1;             // partial row: 24 projections + sum of squares
constexpr int RED_FLOATS = NW * TOK * RS;    // [warp][token][RS], two buffers (tiles alternate)
constexpr int SMEM = STAGES * STAGE_BYTES + 2 * RED_FLOATS * 4 + TOK * 16 * 4 + STAGES * 8 + 16 + 128;
// named barriers (0 is __syncthreads): main warps only; logits full; logits empty
constexpr int BAR_MAIN = 1, BAR_FULL = 2, BAR_EMPTY = 3;
}  // namespace map_pipe

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}
// packed pairs of floats (lo in the low word) for the f32x2 pipe
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(lo), "=f"(hi) : "l"(v));
  return make_float2(lo, hi);
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// a 16-bit pair (lo in the low half) as a packed float pair
template <typename T16>
__device__ __forceinline__ uint64_t f2from16(uint32_t w) {
  const float2 f = unpack2<T16>(w);
  return f2pack(f.x, f.y);
}
template <>
__device__ __forceinline__ uint64_t f2from16<__nv_bfloat16>(uint32_t w) {
  // a bfloat16 is the upper half of the float with the same value
  return (uint64_t)(w << 16) | ((uint64_t)(w & 0xffff0000u) << 32);
}
// a packed float pair rounded to a 16-bit pair (fp16: saturating, as from_f)
template <typename TU>
__device__ __forceinline__ uint32_t f2to16(uint64_t v) {
  const float2 f = f2unpack(v);
  return pack2<TU>(f.x, f.y);
}
template <>
__device__ __forceinline__ uint32_t f2to16<float>(uint64_t) { return 0; }  // not used (u is 16-bit here)

// named barrier that also returns whether any participating thread passed p
__device__ __forceinline__ bool named_sync_or(int id, int n, bool p) {
  uint32_t r;
  asm volatile(
      "{\n"
      ".reg .pred pi, po;\n"
      "setp.ne.u32 pi, %1, 0;\n"
      "bar.red.or.pred po, %2, %3, pi;\n"
      "selp.u32 %0, 1, 0, po;\n"
      "}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

template <typename TX, typename TU>
__global__ void __launch_bounds__(map_pipe::THREADS, 1)
mhc_map_pipe_kernel(const TX* __restrict__ x, int64_t ntok, const uint2* __restrict__ phif,
                    const float* __restrict__ mp, float map_eps, const float* __restrict__ norm_w, float norm_eps,
                    TU* __restrict__ u, float* __restrict__ hmix) {
  using namespace map_pipe;
  constexpr int KS = D / 16 / NW;  // k-steps per warp (8)
  constexpr int VPL = C / 256;     // 16-byte chunks per lane and stream row
  constexpr int MT = NW * 32;      // main threads
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* ring = smem_raw;
  float* red = reinterpret_cast<float*>(ring + STAGES * STAGE_BYTES);  // [NW][TOK][RS]
  float* hres = red + 2 * RED_FLOATS;                                  // [TOK][16] H_res logits
  uint64_t* bar = reinterpret_cast<uint64_t*>(hres + TOK * 16);        // [STAGES] stage full
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + STAGES);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int64_t ntiles = (ntok + TOK - 1) / TOK;
  if (tid == 0) {
    for (int st = 0; st < STAGES; ++st) tc05::mbar_init(bar + st, NW);  // one arrival per main warp
    tc05::fence_barrier_init();
    *abort_flag = 0;
  }
  __syncthreads();
  // main warp w fills row w of stage st with its token of the tile (one
  // arrival per warp; rows past ntok arrive without a copy and keep stale
  // values, whose results are never stored); lane 0 calls it
  auto load_row = [&](int st, int64_t tile, int w) {
    const int64_t tk = tile * TOK + w;
    if (tk < ntok) {
      tc05::mbar_arrive_expect_tx(bar + st, (uint32_t)(D * 2));
      tc05::bulk_load(ring + st * STAGE_BYTES + w * ROWB, x + tk * D, D * 2, bar + st);
    } else {
      tc05::mbar_arrive(bar + st);
    }
  };

  if (warp == NW) {
    // ---- the Sinkhorn warp
    named_arrive(BAR_EMPTY, THREADS);  // the logits buffer starts empty
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      named_sync(BAR_FULL, THREADS);
      if (*abort_flag) return;
      float M[16];
      if (lane < TOK) {
#pragma unroll
        for (int q = 0; q < 16; ++q) M[q] = hres[lane * 16 + q];
      }
      // the main warps wait for this before writing the next tile's logits
      // (no arrival after the last tile: every barrier phase completes)
      if (tile + gridDim.x < ntiles) named_arrive(BAR_EMPTY, THREADS);
      const int64_t tk = tile * TOK + lane;
      if (lane < TOK && tk < ntok) {
        sinkhorn4(M, 20, 1e-8f);
        float4* hd = reinterpret_cast<float4*>(hmix + tk * kMapRows + 8);
#pragma unroll
        for (int q = 0; q < 4; ++q) hd[q] = make_float4(M[4 * q], M[4 * q + 1], M[4 * q + 2], M[4 * q + 3]);
      }
    }
    return;
  }

  // ---- the main warps
#pragma unroll
  for (int st = 0; st < STAGES; ++st) {
    const int64_t t0 = blockIdx.x + (int64_t)st * gridDim.x;
    if (lane == 0 && t0 < ntiles) load_row(st, t0, warp);
  }
  // this warp's phi fragments: its column slice is the same for every tile,
  // so they are loaded once and stay in registers
  uint2 fr[KS][3];
#pragma unroll
  for (int j = 0; j < KS; ++j) {
    const uint2* fp = phif + ((size_t)(warp * KS + j) * 32 + lane) * 3;
    fr[j][0] = __ldg(fp);
    fr[j][1] = __ldg(fp + 1);
    fr[j][2] = __ldg(fp + 2);
  }
  // lane constants of step 2 (lane v serves partial index v of the warp's token)
  const float a_pre = __ldg(mp + 0), a_post = __ldg(mp + 1), a_res = __ldg(mp + 2);
  const float b_lane = lane < 4 ? __ldg(mp + 4 + lane)
                                : (lane < 8 ? __ldg(mp + 8 + (lane - 4)) : (lane < 24 ? __ldg(mp + 12 + (lane - 8)) : 0.f));
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int st = it % STAGES;
    const int64_t tok0 = tile * TOK;
    const unsigned char* xs = ring + st * STAGE_BYTES;
    const bool ok = tc05::mbar_wait(bar + st, (uint32_t)(it / STAGES) & 1u);
    float* redb = red + (it & 1) * RED_FLOATS;  // this tile's partials buffer
    // 1. partial projections over this warp's columns
    float acc[3][4];
#pragma unroll
    for (int n = 0; n < 3; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    float ss_lo = 0.f, ss_hi = 0.f;
    const uint32_t xbase = tc05::smem_u32(xs);
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      const int ks = warp * KS + j;
      const int rr = lane & 15, col = ks * 16 + (lane >> 4) * 8;
      uint32_t a[4];
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                   : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                   : "r"(xbase + (uint32_t)(rr * ROWB + col * 2)));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = unpack2<TX>(a[q]);
        if (q & 1) ss_hi = fmaf(v.x, v.x, fmaf(v.y, v.y, ss_hi));
        else ss_lo = fmaf(v.x, v.x, fmaf(v.y, v.y, ss_lo));
      }
      mma16<TX>(acc[0], a, fr[j][0].x, fr[j][0].y);
      mma16<TX>(acc[1], a, fr[j][1].x, fr[j][1].y);
      mma16<TX>(acc[2], a, fr[j][2].x, fr[j][2].y);
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      ss_lo += __shfl_xor_sync(0xffffffffu, ss_lo, off);
      ss_hi += __shfl_xor_sync(0xffffffffu, ss_hi, off);
    }
    float* rw = redb + warp * TOK * RS;
#pragma unroll
    for (int n = 0; n < 3; ++n) {
      rw[g * RS + 8 * n + 2 * t4] = acc[n][0];
      rw[g * RS + 8 * n + 2 * t4 + 1] = acc[n][1];
      rw[(g + 8) * RS + 8 * n + 2 * t4] = acc[n][2];
      rw[(g + 8) * RS + 8 * n + 2 * t4 + 1] = acc[n][3];
    }
    if (t4 == 0) {
      rw[g * RS + kMapRows] = ss_lo;
      rw[(g + 8) * RS + kMapRows] = ss_hi;
    }
    // partials complete; a stage wait that ran out on any warp aborts all
    if (named_sync_or(BAR_MAIN, MT, !ok)) {
      // release the Sinkhorn warp (its logits-buffer arrival for this tile is
      // in), then wait (bounded) for this CTA's copies in flight
      named_sync(BAR_EMPTY, THREADS);
      if (tid == 0) {
        *abort_flag = 1;
        atomicExch(&g_map_tma_error, (int)WALSH_ERR_TIMEOUT);
      }
      named_arrive(BAR_FULL, THREADS);
      if (tid == 0)
        for (int k = 0; k < STAGES; ++k) {
          const int64_t t2 = tile + (int64_t)k * gridDim.x;
          if (t2 < ntiles) tc05::mbar_wait(bar + (it + k) % STAGES, (uint32_t)((it + k) / STAGES) & 1u, 200000000LL);
        }
      return;
    }

    // 2. this warp's token: lane v < 25 adds partial v over the 16 warps in order
    const int t = warp;
    const int64_t tok = tok0 + t;
    float d = 0.f;
    if (lane < RS) {
#pragma unroll
      for (int w = 0; w < NW; ++w) d += redb[(w * TOK + t) * RS + lane];
    }
    const float rms = rsqrtf(__shfl_sync(0xffffffffu, d, kMapRows) / (float)D + map_eps);
    const float dn = d * rms;
    float hph = 0.f;
    if (lane < 4) hph = 1.0f / (1.0f + expf(-(a_pre * dn + b_lane)));
    else if (lane < 8) hph = 2.0f * (1.0f / (1.0f + expf(-(a_post * dn + b_lane))));
    if (lane < 8 && tok < ntok) hmix[tok * kMapRows + lane] = hph;
    named_sync(BAR_EMPTY, THREADS);  // the Sinkhorn warp has taken the previous tile's logits
    if (lane >= 8 && lane < 24) hres[t * 16 + (lane - 8)] = a_res * dn + b_lane;
    named_arrive(BAR_FULL, THREADS);
    // pre-mix and RMSNorm of the token, its stream rows read from the ring buffer;
    // element pairs on the f32x2 pipe, products and sums in the order of the
    // scalar form ((h0 x0 + h1 x1) + h2 x2) + h3 x3
    {
      const float h0 = __shfl_sync(0xffffffffu, hph, 0), h1 = __shfl_sync(0xffffffffu, hph, 1),
                  h2 = __shfl_sync(0xffffffffu, hph, 2), h3 = __shfl_sync(0xffffffffu, hph, 3);
      const uint64_t h02 = f2pack(h0, h0), h12 = f2pack(h1, h1), h22 = f2pack(h2, h2), h32 = f2pack(h3, h3);
      uint64_t uv[VPL][4];
      uint64_t s2a = f2pack(0.f, 0.f), s2b = s2a;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        uint4 xq[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          xq[jj] = *reinterpret_cast<const uint4*>(xs + t * ROWB + (jj * C + (lane + 32 * v) * 8) * 2);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t w0 = (&xq[0].x)[q], w1 = (&xq[1].x)[q], w2 = (&xq[2].x)[q], w3 = (&xq[3].x)[q];
          uint64_t a = f2mul(h02, f2from16<TX>(w0));
          a = f2fma(h12, f2from16<TX>(w1), a);
          a = f2fma(h22, f2from16<TX>(w2), a);
          a = f2fma(h32, f2from16<TX>(w3), a);
          uv[v][q] = a;
          if (q & 1) s2b = f2fma(a, a, s2b);
          else s2a = f2fma(a, a, s2a);
        }
      }
      const float2 sa = f2unpack(s2a), sb = f2unpack(s2b);
      const float s2 = warp_sum((sa.x + sa.y) + (sb.x + sb.y));
      const float rn = norm_w ? rsqrtf(s2 / (float)C + norm_eps) : 1.0f;
      const uint64_t rn2 = f2pack(rn, rn);
      if (tok < ntok) {
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int cc = (lane + 32 * v) * 8;
          float4 nwa = make_float4(1.f, 1.f, 1.f, 1.f), nwb = nwa;
          if (norm_w) {
            nwa = __ldg(reinterpret_cast<const float4*>(norm_w + cc));
            nwb = __ldg(reinterpret_cast<const float4*>(norm_w + cc + 4));
          }
          const uint64_t nw2[4] = {f2pack(nwa.x, nwa.y), f2pack(nwa.z, nwa.w), f2pack(nwb.x, nwb.y),
                                   f2pack(nwb.z, nwb.w)};
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) w[q] = f2to16<TU>(f2mul(f2mul(uv[v][q], rn2), nw2[q]));
          *reinterpret_cast<uint4*>(u + tok * C + cc) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    // every warp has read the whole stage (phase 1, before the partials
    // barrier) and this warp is done with its row: refill the row with its
    // token of the tile STAGES ahead; the next tile's partials go to the
    // other buffer, so no barrier here
    __syncwarp();
    const int64_t next = tile + (int64_t)STAGES * gridDim.x;
    if (lane == 0 && next < ntiles) {
      tc05::fence_proxy_async();
      load_row(st, next, warp);
    }
  }
}

template <typename T>
__global__ void mhc_post_kernel(const T* x, const T* __restrict__ f, const float* __restrict__ hmix, int64_t ntok,
                                int C, T* xo) {
  const int64_t total = ntok * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / C;
    const int c = (int)(i - tok * C);
    const float* hm = hmix + tok * kMapRows;
    const size_t base = (size_t)tok * 4 * C + c;
    const float x0 = to_f(x[base]), x1 = to_f(x[base + C]), x2 = to_f(x[base + 2 * C]), x3 = to_f(x[base + 3 * C]);
    const float fv = to_f(f[i]);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float* hr = hm + 8 + 4 * r;
      const float v = (((hr[0] * x0 + hr[1] * x1) + hr[2] * x2) + hr[3] * x3) + hm[4 + r] * fv;
      xo[base + (size_t)r * C] = from_f<T>(v);
    }
  }
}

__global__ void sinkhorn_kernel(const float* __restrict__ h, int64_t n, int iters, float eps, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float M[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) M[k] = h[i * 16 + k];
    sinkhorn4(M, iters, eps);
#pragma unroll
    for (int k = 0; k < 16; ++k) out[i * 16 + k] = M[k];
  }
}

template <typename T, typename TU, int TPW>
static int launch_map(const void* x, int64_t ntok, int C, const float* phi, const float* mp, float map_eps,
                      const float* norm_w, float norm_eps, void* u, float* hmix, cudaStream_t s) {
  const size_t smem = (kMapRows * 128 + 8 * TPW * kMapRows + 8 * C) * sizeof(float);
  auto kern = mhc_map_kernel<T, TU, TPW>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (ntok + 8 * TPW - 1) / (8 * TPW);
  kern<<<(unsigned)grid, 256, smem, s>>>((const T*)x, ntok, C, phi, mp, map_eps, norm_w, norm_eps, (TU*)u, hmix);
  return launch_status();
}

static inline int grid_for(int64_t total, int threads) {
  int64_t g = (total + threads - 1) / threads;
  return (int)(g < 148 * 16 ? (g < 1 ? 1 : g) : 148 * 16);
}

}  // namespace walsh

using namespace walsh;

template <int C, typename TX, typename TU, int TOKN>
static int launch_map_tma_n(const void* x, int64_t ntok, const void* phi_frag, const float* mp, float map_eps,
                            const float* norm_w, float norm_eps, void* u, float* hmix, cudaStream_t s);

// Single-pass TMA kernel launch; 1 = ran, 0 = not applicable, < 0 = error.
template <int C, typename TX, typename TU>
static int launch_map_tma(const void* x, int64_t ntok, const void* phi_frag, const float* mp, float map_eps,
                          const float* norm_w, float norm_eps, void* u, float* hmix, cudaStream_t s) {
  // 8 tokens per CTA for C = 2048, and for C = 512 while 16-token CTAs
  // would not fill the SMs
  if constexpr (C == 512) {
    if (ntok > 148 * 16)
      return launch_map_tma_n<C, TX, TU, 16>(x, ntok, phi_frag, mp, map_eps, norm_w, norm_eps, u, hmix, s);
  }
  return launch_map_tma_n<C, TX, TU, 8>(x, ntok, phi_frag, mp, map_eps, norm_w, norm_eps, u, hmix, s);
}

template <int C, typename TX, typename TU, int TOKN>
static int launch_map_tma_n(const void* x, int64_t ntok, const void* phi_frag, const float* mp, float map_eps,
                            const float* norm_w, float norm_eps, void* u, float* hmix, cudaStream_t s) {
  using G = MapTma<C, TOKN>;
  if (ntok > 2147483647LL) return 0;
  CUtensorMap m;
  if (!make_tile_map(&m, x, std::is_same<TX, __nv_bfloat16>::value, ntok, G::D, G::BOXC, G::TOK)) return 0;
  auto kern = mhc_map_tma_kernel<C, TX, TU, TOKN>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM) != cudaSuccess)
    return launch_status();
  kern<<<(unsigned)((ntok + G::TOK - 1) / G::TOK), 256, G::SMEM, s>>>(m, ntok, (const uint2*)phi_frag, mp, map_eps,
                                                                      norm_w, norm_eps, (TU*)u, hmix);
  const int st = launch_status();
  return st == WALSH_OK ? 1 : st;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      n = v;
    else {
      cudaGetLastError();
      return 148;
    }
  }
  return n;
}

// Persistent pipelined kernel for prefill-sized C = 512 calls.
template <typename TX, typename TU>
static int launch_map_pipe(const void* x, int64_t ntok, const void* phi_frag, const float* mp, float map_eps,
                           const float* norm_w, float norm_eps, void* u, float* hmix, cudaStream_t s) {
  using namespace map_pipe;
  auto kern = mhc_map_pipe_kernel<TX, TU>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
    return launch_status();
  const int64_t ntiles = (ntok + TOK - 1) / TOK;
  const int grid = (int)min64(ntiles, num_sms());
  kern<<<grid, THREADS, SMEM, s>>>((const TX*)x, ntok, (const uint2*)phi_frag, mp, map_eps, norm_w, norm_eps,
                                   (TU*)u, hmix);
  return launch_status();
}

// mapping kernel choice for prefill-sized C = 512 calls: 1 = the pipelined
// single-pass kernel (default), 0 = the two-pass tensor-core kernel
static int g_map_pipe = 1;
extern "C" int walsh_map_set_pipe(int on) {
  const int old = g_map_pipe;
  if (on >= 0) g_map_pipe = on ? 1 : 0;
  return old;
}

extern "C" walsh_status walsh_mhc_map(const void* x, int dtype, int64_t ntok, int C, const float* phi,
                                      const void* phi_lp, const void* phi_frag, const float* mparams,
                                      float map_eps, const float* norm_w, float norm_eps, void* u, int u_dtype,
                                      float* hmix, void* stream) {
  if (int e = injected("mhc_map")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_DTYPE(u_dtype);
  WALSH_CHECK_ARG(x && phi && mparams && u && hmix);
  WALSH_CHECK_SHAPE(ntok >= 0 && C > 0 && C % 32 == 0 && C <= 8192);
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // single-pass kernel: 16 tokens per CTA (8 for C = 2048) with its load
  // exposed per CTA; it wins at decode token counts (measured 190 us vs 145 us
  // for the two-pass kernel at 65 536 tokens), so prefill-sized calls take the
  // 128-token two-pass kernel below
  const bool many = ntok >= 148 * 64;
  if (!many && phi_frag && (C == 512 || C == 2048) && (dtype == WALSH_BF16 || dtype == WALSH_F16) &&
      u_dtype != WALSH_F32 && ((((uintptr_t)x) | ((uintptr_t)u) | ((uintptr_t)phi_frag)) & 15u) == 0) {
    int r;
#define WALSH_MAP_TMA(CC)                                                                                        \
  if (dtype == WALSH_BF16)                                                                                      \
    r = u_dtype == WALSH_F16 ? launch_map_tma<CC, __nv_bfloat16, __half>(x, ntok, phi_frag, mparams, map_eps,   \
                                                                         norm_w, norm_eps, u, hmix, s)          \
                             : launch_map_tma<CC, __nv_bfloat16, __nv_bfloat16>(x, ntok, phi_frag, mparams,      \
                                                                                map_eps, norm_w, norm_eps, u,    \
                                                                                hmix, s);                        \
  else                                                                                                          \
    r = u_dtype == WALSH_F16 ? launch_map_tma<CC, __half, __half>(x, ntok, phi_frag, mparams, map_eps, norm_w,   \
                                                                  norm_eps, u, hmix, s)                         \
                             : launch_map_tma<CC, __half, __nv_bfloat16>(x, ntok, phi_frag, mparams, map_eps,    \
                                                                         norm_w, norm_eps, u, hmix, s);
    if (C == 512) {
      WALSH_MAP_TMA(512)
    } else {
      WALSH_MAP_TMA(2048)
    }
#undef WALSH_MAP_TMA
    if (r != 0) return r > 0 ? WALSH_OK : r;
  }
  if (many && g_map_pipe && phi_frag && C == 512 && (dtype == WALSH_BF16 || dtype == WALSH_F16) &&
      u_dtype != WALSH_F32 && ((((uintptr_t)x) | ((uintptr_t)u) | ((uintptr_t)phi_frag)) & 15u) == 0) {
    if (dtype == WALSH_BF16)
      return u_dtype == WALSH_F16
                 ? launch_map_pipe<__nv_bfloat16, __half>(x, ntok, phi_frag, mparams, map_eps, norm_w, norm_eps, u,
                                                          hmix, s)
                 : launch_map_pipe<__nv_bfloat16, __nv_bfloat16>(x, ntok, phi_frag, mparams, map_eps, norm_w,
                                                                 norm_eps, u, hmix, s);
    return u_dtype == WALSH_F16
               ? launch_map_pipe<__half, __half>(x, ntok, phi_frag, mparams, map_eps, norm_w, norm_eps, u, hmix, s)
               : launch_map_pipe<__half, __nv_bfloat16>(x, ntok, phi_frag, mparams, map_eps, norm_w, norm_eps, u,
                                                        hmix, s);
  }
  const bool vec_ok = ((((uintptr_t)x) | ((uintptr_t)u) | ((uintptr_t)phi_lp)) & 15u) == 0;
  // the two-pass tensor-core kernel takes 128 tokens per CTA: below about a
  // wave of those (decode steps), the warp-per-token kernel spreads wider
  if (many && (dtype == WALSH_BF16 || dtype == WALSH_F16) && u_dtype != WALSH_F32 && phi_lp && vec_ok &&
      (C == 512 || C == 2048)) {
    const unsigned grid = (unsigned)((ntok + map_tc::TOK - 1) / map_tc::TOK);
#define WALSH_MAP_TC(CC, TU, TX)                                                                              \
  {                                                                                                          \
    const int smem = (int)map_tc::smem_bytes<CC>();                                                          \
    cudaFuncSetAttribute(mhc_map_mma_kernel<CC, TU, TX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    mhc_map_mma_kernel<CC, TU, TX><<<grid, 256, smem, s>>>((const TX*)x, ntok, (const TX*)phi_lp, mparams,   \
                                                          map_eps, norm_w, norm_eps, (TU*)u, hmix);          \
  }
    const bool uh = u_dtype == WALSH_F16;
    if (dtype == WALSH_BF16) {
      if (C == 512 && uh) WALSH_MAP_TC(512, __half, __nv_bfloat16)
      else if (C == 512) WALSH_MAP_TC(512, __nv_bfloat16, __nv_bfloat16)
      else if (uh) WALSH_MAP_TC(2048, __half, __nv_bfloat16)
      else WALSH_MAP_TC(2048, __nv_bfloat16, __nv_bfloat16)
    } else {
      if (C == 512 && uh) WALSH_MAP_TC(512, __half, __half)
      else if (C == 512) WALSH_MAP_TC(512, __nv_bfloat16, __half)
      else if (uh) WALSH_MAP_TC(2048, __half, __half)
      else WALSH_MAP_TC(2048, __nv_bfloat16, __half)
    }
#undef WALSH_MAP_TC
    return launch_status();
  }
  const bool big = ntok >= 148 * 64;
  return WALSH_DISPATCH_DTYPE(dtype, TX, WALSH_DISPATCH_DTYPE(u_dtype, TU,
      big ? launch_map<TX, TU, 4>(x, ntok, C, phi, mparams, map_eps, norm_w, norm_eps, u, hmix, s)
          : launch_map<TX, TU, 1>(x, ntok, C, phi, mparams, map_eps, norm_w, norm_eps, u, hmix, s)));
}

extern "C" walsh_status walsh_mhc_post(const void* x, const void* f, const float* hmix, int dtype, int64_t ntok,
                                       int C, void* x_out, void* stream) {
  if (int e = injected("mhc_post")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(x && f && hmix && x_out);
  WALSH_CHECK_SHAPE(ntok >= 0 && C > 0);
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int g = grid_for(ntok * C, 256);
  return WALSH_DISPATCH_DTYPE(dtype, T, (mhc_post_kernel<T><<<g, 256, 0, s>>>((const T*)x, (const T*)f, hmix, ntok, C,
                                                                            (T*)x_out), launch_status()));
}

extern "C" walsh_status walsh_sinkhorn(const float* h, int64_t n, int iters, float eps, float* out, void* stream) {
  if (int e = injected("sinkhorn")) return e;
  WALSH_CHECK_ARG(h && out && iters >= 0);
  WALSH_CHECK_SHAPE(n >= 0);
  if (n == 0) return WALSH_OK;
  sinkhorn_kernel<<<grid_for(n, 128), 128, 0, (cudaStream_t)stream>>>(h, n, iters, eps, out);
  return launch_status();
}

extern "C" int walsh_map_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_map_tma_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_map_tma_error, &zero, sizeof(int));
  }
  return v;
}
