// Ternary weights of the .walsh v4 file format on the device.
//
// The file stores a ternary tensor as a bitmask (bit b of byte i: position
// 8 i + b is non-zero) and one sign bit per non-zero in position order (1 =
// +1, 0 = -1) -- compress.py:36-93 writes it, generate_compressed.py:70-105
// reads it one bit at a time on the host.  Here one CTA walks the bitmask in
// 32-bit words: each thread takes a word, an exclusive scan of the words'
// popcounts over the CTA (plus the running count of earlier rounds) gives the
// rank of the word's first non-zero, and each set bit's sign is bit
// (rank + bits below it) of the sign array.  Outputs: the dense values
// (float, row-major) and/or the 2-bit packed layout of this library
// (-1 -> 00, 0 -> 01, +1 -> 10, four per byte along the last dimension k,
// first value in the two most significant bits; the last byte of a row is
// padded with the code of 0).
#include "common.cuh"

namespace walsh {

constexpr int kUnpackThreads = 1024;

__device__ __forceinline__ uint32_t load_word(const uint8_t* p, int64_t word, int64_t nbytes) {
  uint32_t w = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int64_t i = word * 4 + b;
    if (i < nbytes) w |= (uint32_t)p[i] << (8 * b);
  }
  return w;
}

__global__ void __launch_bounds__(kUnpackThreads)
bitmask_ternary_kernel(const uint8_t* __restrict__ mask, int64_t mask_bytes, const uint8_t* __restrict__ signs,
                       int64_t sign_bytes, int64_t total, int64_t nnz, int k, float* __restrict__ dense,
                       uint8_t* __restrict__ packed, int* __restrict__ err) {
  __shared__ int64_t warp_tot[kUnpackThreads / 32];
  __shared__ int64_t base_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nwords = (total + 31) / 32;
  const int kb = (k + 3) / 4;
  if (tid == 0) base_s = 0;
  __syncthreads();
  for (int64_t w0 = 0; w0 < nwords; w0 += kUnpackThreads) {
    const int64_t wi = w0 + tid;
    uint32_t bits = wi < nwords ? load_word(mask, wi, mask_bytes) : 0u;
    if (wi == nwords - 1 && (total & 31)) bits &= (1u << (total & 31)) - 1u;  // bits past the tensor
    const int cnt = __popc(bits);
    // inclusive scan of cnt over the CTA
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int64_t v = lane < kUnpackThreads / 32 ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (lane < kUnpackThreads / 32) warp_tot[lane] = v;  // inclusive per warp
    }
    __syncthreads();
    const int64_t base = base_s;
    const int64_t rank0 = base + (warp > 0 ? warp_tot[warp - 1] : 0) + (incl - cnt);
    if (wi < nwords) {
      int64_t r = rank0;
      for (int b = 0; b < 32; ++b) {
        const int64_t pos = wi * 32 + b;
        if (pos >= total) break;
        float v = 0.f;
        if ((bits >> b) & 1u) {
          int s = 0;
          if (r < nnz && (r >> 3) < sign_bytes) s = (signs[r >> 3] >> (r & 7)) & 1;
          v = s ? 1.f : -1.f;
          ++r;
        }
        if (dense) dense[pos] = v;
      }
    }
    __syncthreads();
    if (tid == kUnpackThreads - 1) base_s = base + warp_tot[kUnpackThreads / 32 - 1];
    __syncthreads();
  }
  if (tid == 0 && base_s != nnz) atomicExch(err, (int)WALSH_ERR_ARG);
  if (!packed) return;
  // pack from the dense values just written (same CTA: visible after the barrier)
  __syncthreads();
  const int64_t rows = total / k;
  for (int64_t i = tid; i < rows * kb; i += kUnpackThreads) {
    const int64_t row = i / kb;
    const int c = (int)(i - row * kb);
    uint32_t byte = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = c * 4 + j;
      const uint32_t code = col < k ? (uint32_t)((int)dense[row * k + col] + 1) : 1u;
      byte |= code << (6 - 2 * j);
    }
    packed[i] = (uint8_t)byte;
  }
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_bitmask_ternary_unpack(const uint8_t* bitmask, int64_t mask_bytes,
                                                     const uint8_t* sign_bits, int64_t sign_bytes, int64_t total,
                                                     int64_t num_nonzero, int k, float* dense, uint8_t* packed,
                                                     int* err, void* stream) {
  if (int e = injected("bitmask_ternary_unpack")) return e;
  WALSH_CHECK_ARG(bitmask && sign_bits && dense && err);
  WALSH_CHECK_SHAPE(total > 0 && k > 0 && total % k == 0 && num_nonzero >= 0 && num_nonzero <= total);
  WALSH_CHECK_SHAPE(mask_bytes >= (total + 7) / 8 && sign_bytes >= (num_nonzero + 7) / 8);
  bitmask_ternary_kernel<<<1, kUnpackThreads, 0, (cudaStream_t)stream>>>(bitmask, mask_bytes, sign_bits, sign_bytes,
                                                                         total, num_nonzero, k, dense, packed, err);
  return launch_status();
}
