// Load-time ternary quantisation / 2-bit packing and the bit-exact unpack.
//
// Quantiser: BitNet b1.58 absmean (src/model/physics.py:13-51,
// src/model/moe.py:268-303): gamma = mean|W| + 1e-8 (float32),
// q = clamp(round_half_even(W / gamma), -1, 1).  Packing follows
// pack_ternary_weights (src/model/fht_cuda.py:65-93).
#include "common.cuh"

namespace walsh {

// One CTA: deterministic double-precision sum of |w|, rounded once to float.
__global__ void __launch_bounds__(1024) absmean_kernel(const float* __restrict__ w, int64_t n,
                                                       float* __restrict__ gamma) {
  __shared__ double part[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += fabs((double)w[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) *gamma = __fadd_rn((float)(v / (double)n), 1e-8f);
  }
}

__global__ void quant_pack_kernel(const float* __restrict__ w, int64_t rows, int k,
                                  const float* __restrict__ gamma, uint8_t* __restrict__ packed) {
  const int kb = (k + 3) >> 2;
  const int64_t total = rows * kb;
  const float g = *gamma;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / kb;
    const int b = (int)(i - r * kb);
    uint32_t byte = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = 4 * b + j;
      int code = 1;  // zero
      if (c < k) {
        float q = rintf(__fdiv_rn(w[r * k + c], g));
        q = fminf(fmaxf(q, -1.0f), 1.0f);
        code = (int)q + 1;
      }
      byte |= (uint32_t)code << (6 - 2 * j);
    }
    packed[i] = (uint8_t)byte;
  }
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int64_t rows, int k,
                              float* __restrict__ out) {
  const int kb = (k + 3) >> 2;
  const int64_t total = rows * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k;
    const int c = (int)(i - r * k);
    out[i] = tern_val(packed[r * kb + (c >> 2)], c & 3);
  }
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_ternary_quantize_pack(const float* w, int64_t rows, int k,
                                                    uint8_t* packed, float* gamma, void* stream) {
  if (int e = injected("ternary_quantize_pack")) return e;
  WALSH_CHECK_ARG(w && packed && gamma);
  WALSH_CHECK_SHAPE(rows > 0 && k > 0);
  cudaStream_t s = (cudaStream_t)stream;
  absmean_kernel<<<1, 1024, 0, s>>>(w, rows * (int64_t)k, gamma);
  const int64_t total = rows * ((k + 3) / 4);
  const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  quant_pack_kernel<<<grid, 256, 0, s>>>(w, rows, k, gamma, packed);
  return launch_status();
}

extern "C" walsh_status walsh_ternary_unpack(const uint8_t* packed, int64_t rows, int k, float* out,
                                             void* stream) {
  if (int e = injected("ternary_unpack")) return e;
  WALSH_CHECK_ARG(packed && out);
  WALSH_CHECK_SHAPE(rows > 0 && k > 0);
  const int64_t total = rows * (int64_t)k;
  const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  unpack_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(packed, rows, k, out);
  return launch_status();
}
