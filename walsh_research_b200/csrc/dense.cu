// Dense helpers around the layer stack: embedding gather, a tiled
// y = x W^T + b kernel (stream_merge, tied logits, load-time folding of
// stream_proj into the embedding table) and the chassis RMSNorm.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "mma.cuh"

namespace walsh {

template <typename T>
__global__ void gather_kernel(const int64_t* __restrict__ idx, int64_t ntok, const T* __restrict__ table, int64_t V,
                              int D, T* __restrict__ out, int* err) {
  const int64_t total = ntok * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / D;
    const int c = (int)(i - t * D);
    const int64_t id = __ldg(idx + t);
    if (id < 0 || id >= V) {
      out[i] = from_f<T>(0.f);
      if (err && c == 0) atomicExch(err, (int)WALSH_ERR_INDEX);
    } else {
      out[i] = table[id * D + c];
    }
  }
}

// Row-vectorised gather (rows of D * sizeof(T) bytes, a multiple of 16, table
// and out 16-byte aligned): one warp per token, the index checked once, the
// row copied as 16-byte vectors (an out-of-range index writes a zero row and
// sets *err, as gather_kernel does).
template <typename T>
__global__ void __launch_bounds__(256)
gather_vec_kernel(const int64_t* __restrict__ idx, int64_t ntok, const T* __restrict__ table, int64_t V, int D,
                  T* __restrict__ out, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarp = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = D * (int)sizeof(T) / 16;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < ntok; t += nwarp) {
    const int64_t id = __ldg(idx + t);
    uint4* dst = reinterpret_cast<uint4*>(out + t * D);
    if (id < 0 || id >= V) {
      for (int v = lane; v < nvec; v += 32) dst[v] = make_uint4(0u, 0u, 0u, 0u);
      if (err && lane == 0) atomicExch(err, (int)WALSH_ERR_INDEX);
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(table + id * D);
      for (int v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
    }
  }
}

// 64x64 output tile per CTA, 4x4 per thread, K staged 16 at a time.
template <typename Tx, typename Tw, typename Ty>
__global__ void __launch_bounds__(256)
linear_kernel(const Tx* __restrict__ x, int64_t M, int K, int64_t ldx, const Tw* __restrict__ w, int64_t N,
              const float* __restrict__ bias, Ty* __restrict__ y) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, kk = i - r * BK;
      const int64_t m = m0 + r, n = n0 + r;
      const int k = k0 + kk;
      xs[kk][r] = (m < M && k < K) ? to_f(x[m * ldx + k]) : 0.f;
      ws[kk][r] = (n < N && k < K) ? to_f(w[n * K + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n < N) y[m * N + n] = from_f<Ty>(acc[i][j] + (bias ? __ldg(bias + n) : 0.f));
    }
  }
}

template <typename T, typename Ty>
__global__ void __launch_bounds__(256)
rmsnorm_kernel(const T* x, int64_t rows, int C, const float* __restrict__ w, float eps, Ty* y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < rows; r += (int64_t)gridDim.x * 8) {
    const T* xr = x + r * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = to_f(xr[c]);
      s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    const float inv = rsqrtf(s / (float)C + eps);
    for (int c = lane; c < C; c += 32) y[r * C + c] = from_f<Ty>(to_f(xr[c]) * inv * __ldg(w + c));
  }
}

// ---------------------------------------------------------------------------
// y = x W^T + b at float32 accuracy on the bf16 tensor cores (stream_merge and
// the tied logits).  W is held as two bf16 matrices, W = W_hi + W_lo
// (W_lo = bf16(W - W_hi)), which together carry 16 significant bits with
// float32's exponent range; a float32 x is split the same way in registers.
// Each product accumulates x_hi W_hi + x_hi W_lo + x_lo W_hi in float32
// (x_lo W_lo, below 2^-16 relative, is dropped); a bf16 x is exact in one
// term.  CTA tile 64 x 128, 8 warps of 32 x 32, K staged 32 wide in a
// 3-stage cp.async pipeline; zero-filled rows past M and N.
// ---------------------------------------------------------------------------
namespace lin_split {
constexpr int BM = 64, BN = 128, BK = 32, STAGES = 3, LD = BK + 8;
template <typename Tx>
constexpr int stage_bytes() { return 2 * BN * LD * 2 + BM * LD * (int)sizeof(Tx); }

__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(a, b);
  const float2 h = unpack2<__nv_bfloat16>(hi);
  lo = pack_bf16(a - h.x, b - h.y);
}
}  // namespace lin_split

template <typename Tx>
__global__ void __launch_bounds__(256)
linear_split_kernel(const Tx* __restrict__ x, int64_t M, int K, int64_t ldx, const __nv_bfloat16* __restrict__ whi,
                    const __nv_bfloat16* __restrict__ wlo, int64_t N, const float* __restrict__ bias,
                    float* __restrict__ y) {
  using namespace lin_split;
  constexpr bool XF = !std::is_same<Tx, __nv_bfloat16>::value;  // float or fp16 x: split into bf16 hi + lo
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int wm = warp & 1, wn = warp >> 1;
  const int nk = K / BK;
  auto Wh = [&](int st) { return reinterpret_cast<__nv_bfloat16*>(smem_raw + st * stage_bytes<Tx>()); };
  auto Wl = [&](int st) { return Wh(st) + BN * LD; };
  auto Xs = [&](int st) { return reinterpret_cast<Tx*>(smem_raw + st * stage_bytes<Tx>() + 2 * BN * LD * 2); };
  auto load_stage = [&](int kt, int st) {
    const int k0 = kt * BK;
    __nv_bfloat16* wh = Wh(st);
    __nv_bfloat16* wl = Wl(st);
    for (int i = tid; i < BN * (BK / 8); i += 256) {
      const int r = i / (BK / 8), c = (i % (BK / 8)) * 8;
      const int64_t n = n0 + r;
      const bool in = n < N;
      const size_t off = (size_t)(in ? n : 0) * K + k0 + c;
      cp_async16(wh + r * LD + c, whi + off, in ? 16 : 0);
      cp_async16(wl + r * LD + c, wlo + off, in ? 16 : 0);
    }
    constexpr int XV = 16 / (int)sizeof(Tx);  // elements per 16-byte chunk
    Tx* xs = Xs(st);
    for (int i = tid; i < BM * (BK / XV); i += 256) {
      const int r = i / (BK / XV), c = (i % (BK / XV)) * XV;
      const int64_t m = m0 + r;
      const bool in = m < M;
      cp_async16(xs + r * LD + c, x + (size_t)(in ? m : 0) * ldx + k0 + c, in ? 16 : 0);
    }
  };
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (st < nk) load_stage(st, st);
    cp_async_commit();
  }
  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;
  for (int kt = 0; kt < nk; ++kt) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (kt + STAGES - 1 < nk) load_stage(kt + STAGES - 1, (kt + STAGES - 1) % STAGES);
    cp_async_commit();
    const int st = kt % STAGES;
    const __nv_bfloat16* wh = Wh(st);
    const __nv_bfloat16* wl = Wl(st);
    const Tx* xs = Xs(st);
#pragma unroll
    for (int kk = 0; kk < BK; kk += 16) {
      uint32_t ah[2][4], al[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int r = wm * 32 + mi * 16;
        if constexpr (XF) {
          auto pair = [&](int idx) -> float2 {
            if constexpr (std::is_same<Tx, float>::value)
              return *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(xs) + idx);
            else
              return unpack2<__half>(*reinterpret_cast<const uint32_t*>(xs + idx));
          };
          const float2 v0 = pair((r + g) * LD + kk + 2 * t4);
          const float2 v1 = pair((r + g + 8) * LD + kk + 2 * t4);
          const float2 v2 = pair((r + g) * LD + kk + 8 + 2 * t4);
          const float2 v3 = pair((r + g + 8) * LD + kk + 8 + 2 * t4);
          split2(v0.x, v0.y, ah[mi][0], al[mi][0]);
          split2(v1.x, v1.y, ah[mi][1], al[mi][1]);
          split2(v2.x, v2.y, ah[mi][2], al[mi][2]);
          split2(v3.x, v3.y, ah[mi][3], al[mi][3]);
        } else {
          ldsm_x4(ah[mi], xs + (r + (lane & 15)) * LD + kk + (lane >> 4) * 8);
        }
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int rn = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int cn = kk + ((lane >> 3) & 1) * 8;
        uint32_t bh[4], bl[4];
        ldsm_x4(bh, wh + rn * LD + cn);
        ldsm_x4(bl, wl + rn * LD + cn);
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float* c = acc[mi][2 * np + h];
            if constexpr (XF) mma_bf16(c, al[mi], bh[2 * h], bh[2 * h + 1]);
            mma_bf16(c, ah[mi], bl[2 * h], bl[2 * h + 1]);
            mma_bf16(c, ah[mi], bh[2 * h], bh[2 * h + 1]);
          }
        }
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      const int64_t n = n0 + wn * 32 + ni * 8 + 2 * t4;
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const int64_t m = m0 + wm * 32 + mi * 16 + g + hrow * 8;
        if (m >= M) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (n + e < N) y[m * N + n + e] = acc[mi][ni][hrow * 2 + e] + (bias ? __ldg(bias + n + e) : 0.f);
      }
    }
}

template <typename Tx, typename Tw, typename Ty>
static int launch_linear(const void* x, int64_t M, int K, int64_t ldx, const void* w, int64_t N, const float* bias,
                         void* y, cudaStream_t s) {
  dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64));
  linear_kernel<Tx, Tw, Ty><<<grid, 256, 0, s>>>((const Tx*)x, M, K, ldx, (const Tw*)w, N, bias, (Ty*)y);
  return launch_status();
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_embed_gather(const int64_t* idx, int64_t ntok, const void* table, int dtype, int64_t V,
                                           int D, void* out, int* err, void* stream) {
  if (int e = injected("embed_gather")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(idx && table && out);
  WALSH_CHECK_SHAPE(ntok >= 0 && V > 0 && D > 0);
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int esz = dtype == WALSH_F32 ? 4 : 2;
  if (((int64_t)D * esz) % 16 == 0 && ((((uintptr_t)table) | ((uintptr_t)out)) & 15u) == 0) {
    int64_t g = (ntok + 7) / 8;  // 8 warps (tokens) per CTA
    if (g > 148 * 16) g = 148 * 16;
    return WALSH_DISPATCH_DTYPE(dtype, T,
                                (gather_vec_kernel<T><<<(unsigned)g, 256, 0, s>>>(idx, ntok, (const T*)table, V, D,
                                                                                  (T*)out, err),
                                 launch_status()));
  }
  int64_t g = (ntok * D + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return WALSH_DISPATCH_DTYPE(dtype, T, (gather_kernel<T><<<(unsigned)g, 256, 0, s>>>(idx, ntok, (const T*)table, V, D,
                                                                                    (T*)out, err),
                                         launch_status()));
}

extern "C" walsh_status walsh_linear_fwd(const void* x, int x_dtype, int64_t M, int K, int64_t ldx, const void* w,
                                         int w_dtype, int64_t N, const float* bias, void* y, int y_dtype,
                                         void* stream) {
  if (int e = injected("linear_fwd")) return e;
  WALSH_CHECK_DTYPE(x_dtype);
  WALSH_CHECK_DTYPE(w_dtype);
  WALSH_CHECK_DTYPE(y_dtype);
  WALSH_CHECK_ARG(x && w && y);
  WALSH_CHECK_SHAPE(M >= 0 && K > 0 && N > 0 && ldx >= K);
  WALSH_CHECK_SHAPE((M + 63) / 64 <= 65535);
  if (M == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  return WALSH_DISPATCH_DTYPE(x_dtype, TX, WALSH_DISPATCH_DTYPE(w_dtype, TW, WALSH_DISPATCH_DTYPE(y_dtype, TY,
      (launch_linear<TX, TW, TY>(x, M, K, ldx, w, N, bias, y, s)))));
}

extern "C" walsh_status walsh_rmsnorm(const void* x, int dtype, int64_t rows, int C, const float* w, float eps,
                                      void* y, int y_dtype, void* stream) {
  if (int e = injected("rmsnorm")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_DTYPE(y_dtype);
  WALSH_CHECK_ARG(x && w && y);
  WALSH_CHECK_SHAPE(rows >= 0 && C > 0);
  if (rows == 0) return WALSH_OK;
  int64_t g = (rows + 7) / 8;
  if (g > 148 * 32) g = 148 * 32;
  cudaStream_t s = (cudaStream_t)stream;
  return WALSH_DISPATCH_DTYPE(dtype, T, WALSH_DISPATCH_DTYPE(y_dtype, TY,
      (rmsnorm_kernel<T, TY><<<(unsigned)g, 256, 0, s>>>((const T*)x, rows, C, w, eps, (TY*)y), launch_status())));
}

namespace walsh {

// The same three-product split on the tcgen05 kernel as ONE GEMM with K
// tripled: [x_hi | x_hi | x_lo] [w_hi | w_lo | w_hi]^T = x_hi w_hi^T +
// x_hi w_lo^T + x_lo w_hi^T, fp32 accumulation, fp32 store.
int gemm_bf16_f32out(const __nv_bfloat16* a, int64_t M, int K, const __nv_bfloat16* w, int64_t N, float* y,
                     cudaStream_t s);  // octonion.cu

__global__ void split3_rows_kernel(const float* __restrict__ x, int64_t M, int K, __nv_bfloat16* __restrict__ a3) {
  const int64_t total = M * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / K;
    const int k = (int)(i - m * K);
    const float v = x[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16* row = a3 + m * 3 * K;
    row[k] = hi;
    row[K + k] = hi;
    row[2 * K + k] = lo;
  }
}

}  // namespace walsh

extern "C" int64_t walsh_linear_split_tc_scratch_bytes(int64_t M, int K) { return (M * 3 * K * 2 + 255) / 256 * 256; }

extern "C" walsh_status walsh_linear_split_tc_fwd(const float* x, int64_t M, int K, const void* w3, int64_t N,
                                                  void* scratch, float* y, void* stream) {
  using namespace walsh;
  if (int e = injected("linear_split_tc_fwd")) return e;
  WALSH_CHECK_ARG(x && w3 && scratch && y);
  WALSH_CHECK_SHAPE(M >= 0 && K > 0 && N > 0 && K % 8 == 0 && M <= 2147483647LL && N <= 2147483647LL);
  if ((((uintptr_t)x) | ((uintptr_t)w3) | ((uintptr_t)scratch)) & 15u) return WALSH_ERR_ALIGN;
  if (M == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  __nv_bfloat16* a3 = reinterpret_cast<__nv_bfloat16*>(scratch);
  const unsigned g = (unsigned)std::min<int64_t>((M * K + 255) / 256, 148 * 16);
  split3_rows_kernel<<<g, 256, 0, s>>>(x, M, K, a3);
  if (int e = launch_status()) return e;
  return gemm_bf16_f32out(a3, M, 3 * K, reinterpret_cast<const __nv_bfloat16*>(w3), N, y, s);
}

extern "C" walsh_status walsh_linear_split_fwd(const void* x, int x_dtype, int64_t M, int K, int64_t ldx,
                                               const void* w_hi, const void* w_lo, int64_t N, const float* bias,
                                               float* y, void* stream) {
  using namespace lin_split;
  if (int e = injected("linear_split_fwd")) return e;
  WALSH_CHECK_DTYPE(x_dtype);
  WALSH_CHECK_ARG(x && w_hi && w_lo && y);
  WALSH_CHECK_SHAPE(M >= 0 && K > 0 && N > 0 && ldx >= K && K % BK == 0);
  WALSH_CHECK_SHAPE((N + BN - 1) / BN <= 65535);
  const int esz = x_dtype == WALSH_F32 ? 4 : 2;
  if ((((uintptr_t)x) | ((uintptr_t)w_hi) | ((uintptr_t)w_lo)) & 15u) return WALSH_ERR_ALIGN;
  if ((ldx * esz) % 16) return WALSH_ERR_ALIGN;
  if (M == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  auto go = [&](auto kernel, int smem, auto xp) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return launch_status();
    kernel<<<grid, 256, smem, s>>>(xp, M, K, ldx, (const __nv_bfloat16*)w_hi, (const __nv_bfloat16*)w_lo, N, bias,
                                   y);
    return launch_status();
  };
  if (x_dtype == WALSH_F32)
    return go(linear_split_kernel<float>, STAGES * stage_bytes<float>(), (const float*)x);
  if (x_dtype == WALSH_F16)
    return go(linear_split_kernel<__half>, STAGES * stage_bytes<__half>(), (const __half*)x);
  return go(linear_split_kernel<__nv_bfloat16>, STAGES * stage_bytes<__nv_bfloat16>(), (const __nv_bfloat16*)x);
}
