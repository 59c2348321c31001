// Dense helpers around the layer stack: embedding gather, a tiled
// y = x W^T + b kernel (stream_merge, tied logits, load-time folding of
// stream_proj into the embedding table) and the chassis RMSNorm.
#include "common.cuh"

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
  int64_t g = (ntok * D + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  cudaStream_t s = (cudaStream_t)stream;
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
