// Hadamard-32 algebra kernels: HadamardLinear, fused q/k/v + RoPE + KV write,
// and Hadamard head mixing.
//
// HadamardLinear (src/model/fht_cuda.py:489-519) computes, per token,
//   y[h, o] = beta[h, o] * sum_g H[g, h] * sum_i W[g, o, i] * sum_g' H[g', g] * alpha[g', i] * x[g', i]
// with H the normalised Sylvester matrix.  Both H products are applied here as
// unnormalised in-register butterflies (fht32) and the two 1/sqrt(32)
// factors are folded into one 1/32 in the epilogue.
//
// Tile layout: a CTA owns TM tokens.  The token tile lives in shared memory
// as float [TM][32][IN_O]; phase 1 (alpha + butterflies over g) gives one
// thread per (token, i) column, phase 2 (the 32 independent ternary
// [OUT_O x IN_O] mat-vecs) one thread per (g, 4 consecutive o), phase 3
// (butterflies over h) one thread per (token, o) column, and the epilogue
// writes coalesced rows.  Ternary weights are read 2 bits at a time from the
// packed tensor (one 32-bit word per weight row for IN_O = 16).
#include "common.cuh"

namespace walsh {

struct QkvEpilogue {
  int T, n_head, hd, ctx, start_pos;
  const float* cos;  // [n_pos, hd/2]
  const float* sin;
};

template <int IN_O, int OUT_O>
struct HCfg {
  static constexpr int TM = (IN_O >= 64 || OUT_O >= 64) ? 4 : 16;
  static constexpr int KB = (IN_O + 3) / 4;
  static constexpr int XS = TM * 32 * IN_O;
  static constexpr int YS = TM * 32 * OUT_O;
  static constexpr int QUADS = 8 * OUT_O;  // (g, o-quad) work items
  static constexpr int QPT = QUADS >= 256 ? QUADS / 256 : 1;
  static constexpr int TSPLIT = QUADS >= 256 ? 1 : 256 / QUADS;
  static constexpr int TPT = TM / TSPLIT;  // tokens per thread in phase 2
  static_assert(TM % TSPLIT == 0, "token split");
};

// Phase 1 / 3: in-place butterflies over the 32 groups of each column.
template <int W, int TM>
__device__ __forceinline__ void fht_columns(float* s) {
  for (int col = threadIdx.x; col < TM * W; col += blockDim.x) {
    const int t = col / W, i = col - t * W;
    float* base = s + t * 32 * W + i;
    float v[32];
#pragma unroll
    for (int g = 0; g < 32; ++g) v[g] = base[g * W];
    fht32(v);
#pragma unroll
    for (int g = 0; g < 32; ++g) base[g * W] = v[g];
  }
}

// Phase 2 for packed ternary weights W[g][o][i] (2 bits each).
template <int IN_O, int OUT_O>
__device__ __forceinline__ void ternary_matvec(const float* xs, float* ys, const uint8_t* __restrict__ wp,
                                               int ntile) {
  using C = HCfg<IN_O, OUT_O>;
  const int tid = threadIdx.x;
#pragma unroll
  for (int qq = 0; qq < C::QPT; ++qq) {
    const int item = (C::QUADS >= 256) ? (tid + qq * 256) : (tid % C::QUADS);
    const int tpart = (C::QUADS >= 256) ? 0 : (tid / C::QUADS);
    const int g = item / (OUT_O / 4);
    const int o0 = (item - g * (OUT_O / 4)) * 4;
    float acc[C::TPT][4];
#pragma unroll
    for (int t = 0; t < C::TPT; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[t][r] = 0.f;
    const uint8_t* wrow = wp + ((size_t)g * OUT_O + o0) * C::KB;
#pragma unroll 4
    for (int ib = 0; ib < C::KB; ++ib) {
      float w[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t byte = __ldg(wrow + r * C::KB + ib);
#pragma unroll
        for (int j = 0; j < 4; ++j) w[r][j] = tern_val(byte, j);
      }
#pragma unroll
      for (int t = 0; t < C::TPT; ++t) {
        const int tt = tpart * C::TPT + t;
        const float* xp = xs + tt * 32 * IN_O + g * IN_O + ib * 4;
        float xv[4];
        if (IN_O % 4 == 0) {
          const float4 v4 = *reinterpret_cast<const float4*>(xp);
          xv[0] = v4.x; xv[1] = v4.y; xv[2] = v4.z; xv[3] = v4.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) xv[j] = (ib * 4 + j < IN_O) ? xp[j] : 0.f;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[t][r] = fmaf(w[r][j], xv[j], acc[t][r]);
      }
    }
#pragma unroll
    for (int t = 0; t < C::TPT; ++t) {
      const int tt = tpart * C::TPT + t;
      float* yp = ys + tt * 32 * OUT_O + g * OUT_O + o0;
#pragma unroll
      for (int r = 0; r < 4; ++r) yp[r] = acc[t][r];
    }
  }
  (void)ntile;
}

// Loads x (optionally scaled by alpha[c]) into a float tile; rows beyond ntile are zero.
template <int W, int TM, typename Tin>
__device__ __forceinline__ void load_tile(const Tin* __restrict__ x, int64_t t0, int ntile, float* s,
                                          const float* __restrict__ alpha) {
  constexpr int ROW = 32 * W;
  for (int i = threadIdx.x; i < TM * ROW; i += blockDim.x) {
    const int t = i / ROW, c = i - t * ROW;
    float v = 0.f;
    if (t < ntile) {
      v = to_f(x[(t0 + t) * ROW + c]);
      if (alpha) v *= __ldg(alpha + c);
    }
    s[i] = v;
  }
}

// ---------------------------------------------------------------------------
// HadamardLinear
// ---------------------------------------------------------------------------
template <int IN_O, int OUT_O, typename Tin, typename Tout>
__global__ void __launch_bounds__(256)
hlin_kernel(const Tin* __restrict__ x, int64_t ntok, const uint8_t* __restrict__ wp, float out_scale,
            const float* __restrict__ alpha, const float* __restrict__ beta, Tout* __restrict__ y) {
  using C = HCfg<IN_O, OUT_O>;
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  float* ys = xs + C::XS;
  const int64_t t0 = (int64_t)blockIdx.x * C::TM;
  const int ntile = (int)min64(C::TM, ntok - t0);
  load_tile<IN_O, C::TM>(x, t0, ntile, xs, alpha);
  __syncthreads();
  fht_columns<IN_O, C::TM>(xs);
  __syncthreads();
  ternary_matvec<IN_O, OUT_O>(xs, ys, wp, ntile);
  __syncthreads();
  fht_columns<OUT_O, C::TM>(ys);
  __syncthreads();
  constexpr int ROW = 32 * OUT_O;
  for (int i = threadIdx.x; i < ntile * ROW; i += blockDim.x) {
    const int t = i / ROW, c = i - t * ROW;
    y[(t0 + t) * ROW + c] = from_f<Tout>(ys[i] * __ldg(beta + c) * out_scale);
  }
}

// ---------------------------------------------------------------------------
// Fused q/k/v (+ RoPE on q, k) with direct writes into q [B,H,T,hd] and the
// KV caches [B,H,ctx,hd].  The raw token tile is loaded once and re-scaled by
// each projection's alpha.
// ---------------------------------------------------------------------------
template <int IO, typename TI, typename T>
__global__ void __launch_bounds__(256)
qkv_kernel(const TI* __restrict__ u, int64_t ntok, const uint8_t* __restrict__ wq,
           const uint8_t* __restrict__ wk, const uint8_t* __restrict__ wv, const float* __restrict__ aq,
           const float* __restrict__ ak, const float* __restrict__ av, const float* __restrict__ bq,
           const float* __restrict__ bk, const float* __restrict__ bv, T* __restrict__ q,
           T* __restrict__ kc, T* __restrict__ vc, QkvEpilogue ep) {
  using C = HCfg<IO, IO>;
  constexpr int ROW = 32 * IO;
  extern __shared__ float4 smem4[];
  float* xr = reinterpret_cast<float*>(smem4);
  float* xs = xr + C::XS;
  float* ys = xs + C::XS;
  const int64_t t0 = (int64_t)blockIdx.x * C::TM;
  const int ntile = (int)min64(C::TM, ntok - t0);
  load_tile<IO, C::TM>(u, t0, ntile, xr, nullptr);
  const int half = ep.hd >> 1;
#pragma unroll 1
  for (int set = 0; set < 3; ++set) {
    const float* al = set == 0 ? aq : (set == 1 ? ak : av);
    const float* be = set == 0 ? bq : (set == 1 ? bk : bv);
    const uint8_t* wp = set == 0 ? wq : (set == 1 ? wk : wv);
    __syncthreads();
    for (int i = threadIdx.x; i < C::XS; i += blockDim.x) xs[i] = xr[i] * __ldg(al + (i % ROW));
    __syncthreads();
    fht_columns<IO, C::TM>(xs);
    __syncthreads();
    ternary_matvec<IO, IO>(xs, ys, wp, ntile);
    __syncthreads();
    fht_columns<IO, C::TM>(ys);
    __syncthreads();
    // epilogue: one thread per (token, channel pair)
    for (int i = threadIdx.x; i < ntile * (ROW / 2); i += blockDim.x) {
      const int t = i / (ROW / 2);
      const int c = (i - t * (ROW / 2)) * 2;
      const int64_t tok = t0 + t;
      const int b = (int)(tok / ep.T), tt = (int)(tok - (int64_t)b * ep.T);
      const int pos = ep.start_pos + tt;  // cache position; RoPE row is tt (table pre-offset by the caller)
      float v0 = ys[t * ROW + c] * __ldg(be + c) * (1.0f / 32.0f);
      float v1 = ys[t * ROW + c + 1] * __ldg(be + c + 1) * (1.0f / 32.0f);
      const int head = c / ep.hd, d = c - head * ep.hd;
      if (set < 2) {  // RoPE on interleaved (even, odd) pairs
        const float cs = __ldg(ep.cos + (size_t)tt * half + (d >> 1));
        const float sn = __ldg(ep.sin + (size_t)tt * half + (d >> 1));
        const float r0 = v0 * cs - v1 * sn, r1 = v0 * sn + v1 * cs;
        v0 = r0; v1 = r1;
      }
      size_t off;
      T* dst;
      if (set == 0) {
        off = (((size_t)b * ep.n_head + head) * ep.T + tt) * ep.hd + d;
        dst = q;
      } else {
        off = (((size_t)b * ep.n_head + head) * ep.ctx + pos) * ep.hd + d;
        dst = set == 1 ? kc : vc;
      }
      dst[off] = from_f<T>(v0);
      dst[off + 1] = from_f<T>(v1);
    }
  }
}

// ---------------------------------------------------------------------------
// Hadamard head mixer: per token and per group of 32 heads,
//   y[g', o] = beta[o] * sum_h H[h, g'] sum_i W[h, i, o] sum_h' H[h', h] x[h', i]
// (src/model/fht_cuda.py:652-670).  Work unit = (token, head group).
// ---------------------------------------------------------------------------
template <int HD, typename T>
__global__ void __launch_bounds__(256)
headmix_kernel(const T* __restrict__ x, int64_t nunits, const float* __restrict__ W,
               const float* __restrict__ beta, T* __restrict__ y) {
  constexpr int TM = HD >= 32 ? 8 : 16;
  constexpr int ROW = 32 * HD;
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  float* ys = xs + TM * ROW;
  const int64_t u0 = (int64_t)blockIdx.x * TM;
  const int ntile = (int)min64(TM, nunits - u0);
  load_tile<HD, TM>(x, u0, ntile, xs, nullptr);
  __syncthreads();
  fht_columns<HD, TM>(xs);
  __syncthreads();
  // y[t][h][o] = sum_i xs[t][h][i] * W[h][i][o]; thread per (h, o) pair, loop tokens
  for (int item = threadIdx.x; item < 32 * HD; item += blockDim.x) {
    const int h = item / HD, o = item - h * HD;
    float w[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) w[i] = __ldg(W + ((size_t)h * HD + i) * HD + o);
    for (int t = 0; t < TM; ++t) {
      const float* xp = xs + t * ROW + h * HD;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < HD; ++i) acc = fmaf(xp[i], w[i], acc);
      ys[t * ROW + h * HD + o] = acc;
    }
  }
  __syncthreads();
  fht_columns<HD, TM>(ys);
  __syncthreads();
  for (int i = threadIdx.x; i < ntile * ROW; i += blockDim.x) {
    const int t = i / ROW, c = i - t * ROW;
    y[(u0 + t) * ROW + c] = from_f<T>(ys[i] * __ldg(beta + (c % HD)) * (1.0f / 32.0f));
  }
}

template <int IN_O, int OUT_O, typename Tin, typename Tout>
static int launch_hlin(const void* x, int64_t ntok, const uint8_t* wp, float out_scale,
                       const float* alpha, const float* beta, void* y, cudaStream_t s) {
  using C = HCfg<IN_O, OUT_O>;
  const size_t smem = (C::XS + C::YS) * sizeof(float);
  auto kern = hlin_kernel<IN_O, OUT_O, Tin, Tout>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (ntok + C::TM - 1) / C::TM;
  kern<<<(unsigned)grid, 256, smem, s>>>((const Tin*)x, ntok, wp, out_scale, alpha, beta, (Tout*)y);
  return launch_status();
}

template <int IN_O, int OUT_O>
static int dispatch_hlin(const void* x, int xd, int64_t ntok, const uint8_t* wp, float out_scale,
                         const float* alpha, const float* beta, void* y, int yd, cudaStream_t s) {
  return WALSH_DISPATCH_DTYPE(xd, TX, WALSH_DISPATCH_DTYPE(yd, TY,
      (launch_hlin<IN_O, OUT_O, TX, TY>(x, ntok, wp, out_scale, alpha, beta, y, s))));
}

template <int IO, typename TI, typename T>
static int launch_qkv(const void* u, int64_t ntok, const uint8_t* const* w, const float* const* a,
                      const float* const* b, void* q, void* kc, void* vc, QkvEpilogue ep, cudaStream_t s) {
  using C = HCfg<IO, IO>;
  const size_t smem = (2 * C::XS + C::YS) * sizeof(float);
  auto kern = qkv_kernel<IO, TI, T>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (ntok + C::TM - 1) / C::TM;
  kern<<<(unsigned)grid, 256, smem, s>>>((const TI*)u, ntok, w[0], w[1], w[2], a[0], a[1], a[2], b[0], b[1],
                                         b[2], (T*)q, (T*)kc, (T*)vc, ep);
  return launch_status();
}

template <int HD, typename T>
static int launch_headmix(const void* x, int64_t nunits, const float* W, const float* beta, void* y,
                          cudaStream_t s) {
  constexpr int TM = HD >= 32 ? 8 : 16;
  const size_t smem = 2 * TM * 32 * HD * sizeof(float);
  auto kern = headmix_kernel<HD, T>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (nunits + TM - 1) / TM;
  kern<<<(unsigned)grid, 256, smem, s>>>((const T*)x, nunits, W, beta, (T*)y);
  return launch_status();
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_hadamard_linear_fwd(const void* x, int x_dtype, int64_t ntok, int in_o,
                                                  int out_o, const uint8_t* w2bit, float w_scale,
                                                  const float* alpha, const float* beta, void* y,
                                                  int y_dtype, void* stream) {
  if (int e = injected("hadamard_linear_fwd")) return e;
  WALSH_CHECK_DTYPE(x_dtype);
  WALSH_CHECK_DTYPE(y_dtype);
  WALSH_CHECK_ARG(x && w2bit && alpha && beta && y);
  WALSH_CHECK_SHAPE(ntok >= 0);
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const float sc = w_scale / 32.0f;
  if (in_o == 16 && out_o == 16) return dispatch_hlin<16, 16>(x, x_dtype, ntok, w2bit, sc, alpha, beta, y, y_dtype, s);
  if (in_o == 64 && out_o == 64) return dispatch_hlin<64, 64>(x, x_dtype, ntok, w2bit, sc, alpha, beta, y, y_dtype, s);
  if (in_o == 16 && out_o == 64) return dispatch_hlin<16, 64>(x, x_dtype, ntok, w2bit, sc, alpha, beta, y, y_dtype, s);
  if (in_o == 64 && out_o == 16) return dispatch_hlin<64, 16>(x, x_dtype, ntok, w2bit, sc, alpha, beta, y, y_dtype, s);
  return WALSH_ERR_SHAPE;
}

extern "C" walsh_status walsh_attn_qkv_fwd(const void* u, int dtype, int B, int T, int C, int n_head,
                                           const uint8_t* wq_2bit, const float* wq_alpha, const float* wq_beta,
                                           const uint8_t* wk_2bit, const float* wk_alpha, const float* wk_beta,
                                           const uint8_t* wv_2bit, const float* wv_alpha, const float* wv_beta,
                                           const float* rope_cos, const float* rope_sin, int n_pos,
                                           int start_pos, void* q, void* k_cache, void* v_cache, int ctx,
                                           int out_dtype, void* stream) {
  if (int e = injected("attn_qkv_fwd")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_DTYPE(out_dtype);
  WALSH_CHECK_ARG(u && wq_2bit && wq_alpha && wq_beta && wk_2bit && wk_alpha && wk_beta && wv_2bit &&
                  wv_alpha && wv_beta && rope_cos && rope_sin && q && k_cache && v_cache);
  WALSH_CHECK_SHAPE(B > 0 && T > 0 && n_head > 0 && C % n_head == 0 && C % 32 == 0);
  const int hd = C / n_head;
  WALSH_CHECK_SHAPE(hd % 2 == 0 && start_pos >= 0 && start_pos + T <= ctx && T <= n_pos);
  QkvEpilogue ep{T, n_head, hd, ctx, start_pos, rope_cos, rope_sin};
  const uint8_t* w[3] = {wq_2bit, wk_2bit, wv_2bit};
  const float* a[3] = {wq_alpha, wk_alpha, wv_alpha};
  const float* b[3] = {wq_beta, wk_beta, wv_beta};
  const int64_t ntok = (int64_t)B * T;
  cudaStream_t s = (cudaStream_t)stream;
  const int io = C / 32;
  if (io != 16 && io != 64) return WALSH_ERR_SHAPE;
  return WALSH_DISPATCH_DTYPE(dtype, TI, WALSH_DISPATCH_DTYPE(out_dtype, TO,
      io == 16 ? launch_qkv<16, TI, TO>(u, ntok, w, a, b, q, k_cache, v_cache, ep, s)
               : launch_qkv<64, TI, TO>(u, ntok, w, a, b, q, k_cache, v_cache, ep, s)));
}

extern "C" walsh_status walsh_head_mixer_fwd(const void* x, int dtype, int64_t ntok, int n_head, int hd,
                                             const float* W, const float* beta, void* y, void* stream) {
  if (int e = injected("head_mixer_fwd")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(x && W && beta && y);
  WALSH_CHECK_SHAPE(ntok >= 0 && n_head > 0 && n_head % 32 == 0);
  if (ntok == 0) return WALSH_OK;
  const int64_t units = ntok * (n_head / 32);
  cudaStream_t s = (cudaStream_t)stream;
  if (hd != 16 && hd != 32) return WALSH_ERR_SHAPE;
  return WALSH_DISPATCH_DTYPE(dtype, T, hd == 16 ? launch_headmix<16, T>(x, units, W, beta, y, s)
                                                 : launch_headmix<32, T>(x, units, W, beta, y, s));
}
