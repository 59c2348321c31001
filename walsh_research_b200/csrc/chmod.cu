// Channel modulation (HadamardChannelModulation, src/model/moe.py:681-762,
// as used by mHCLlamaBlock.forward, src/model/mhc.py:528-532).
//
// The block views the stream state [B, T, n, C] as [B*n, T, C]: a "segment"
// is seg_len consecutive rows of the flat [B*T*n, C] tensor.  Three steps:
//   stats: partial sums over row chunks of RMSNorm(x) (chassis RMSNorm with
//          the channel_mod_norm weight), written per (segment, chunk) so the
//          reduction order is fixed;
//   mlp:   bulk mean -> scaled-ternary MLP -> per-(segment, block) scale/shift;
//   apply: out = x + xn + 0.5 * (xn * scale + 0.1 * shift - xn).
#include <algorithm>
#include <atomic>
#include <mutex>

#include <cuda.h>

#include "common.cuh"
#include "mma.cuh"
#include "ctx_cache.h"

namespace walsh {

constexpr int kChunkRows = 64;

template <typename T>
__global__ void __launch_bounds__(256)
chmod_stats_kernel(const T* __restrict__ x, int C, int seg_len, const float* __restrict__ w, float eps,
                   float* __restrict__ partial) {
  __shared__ float inv[kChunkRows];
  const int seg = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int r0 = ch * kChunkRows;
  const int nr = min(kChunkRows, seg_len - r0);
  const int64_t row0 = (int64_t)seg * seg_len + r0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < nr; r += 8) {
    const T* xr = x + (row0 + r) * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = to_f(xr[c]);
      s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    if (lane == 0) inv[r] = w ? rsqrtf(s / (float)C + eps) : 1.0f;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += 256) {
    float acc = 0.f;
    for (int r = 0; r < nr; ++r) acc = fmaf(to_f(x[(row0 + r) * C + c]), inv[r], acc);
    partial[((size_t)seg * nch + ch) * C + c] = w ? acc * __ldg(w + c) : acc;
  }
}

// Vectorised single-pass variant (C a multiple of 256, 16-byte aligned rows):
// each warp takes rows warp, warp + 8, ... of the chunk, keeps a row in
// registers (8 consecutive channels per lane per 256-column pass), forms its
// RMS factor with one warp reduction and accumulates the normalised row; the
// 8 warps' partial sums are combined through shared memory.
template <typename T, int C>
__global__ void __launch_bounds__(256)
chmod_stats_vec_kernel(const T* __restrict__ x, int seg_len, const float* __restrict__ w, float eps,
                       float* __restrict__ partial) {
  constexpr int NP = C / 256;
  __shared__ float red[8][C];
  const int seg = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int r0 = ch * kChunkRows;
  const int nr = min(kChunkRows, seg_len - r0);
  const int64_t row0 = (int64_t)seg * seg_len + r0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc[NP][8];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[p][e] = 0.f;
  // the warp's next row is loaded before the current one is used
  Vec8<T> cur[NP], nxt[NP];
  auto load_row = [&](int r, Vec8<T> (&dst)[NP]) {
    const T* xr = x + (row0 + r) * C;
#pragma unroll
    for (int p = 0; p < NP; ++p) dst[p] = ld_vec8(xr + p * 256 + lane * 8);
  };
  if (warp < nr) load_row(warp, cur);
  for (int r = warp; r < nr; r += 8) {
    if (r + 8 < nr) load_row(r + 8, nxt);
    float v[NP][8];
    float s = 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      unpack_vec8(cur[p], v[p]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[p][e], v[p][e], s);
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) cur[p] = nxt[p];
    s = warp_sum(s);
    const float inv = w ? rsqrtf(s / (float)C + eps) : 1.0f;
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[p][e] = fmaf(v[p][e], inv, acc[p][e]);
  }
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int e = 0; e < 8; ++e) red[warp][p * 256 + lane * 8 + e] = acc[p][e];
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += 256) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][c];
    partial[((size_t)seg * nch + ch) * C + c] = w ? t * __ldg(w + c) : t;
  }
}

// Vectorised apply (C a multiple of 256): warp per row, 8 channels per lane per pass.
template <typename T, int C>
__global__ void __launch_bounds__(256)
chmod_apply_vec_kernel(const T* x, int64_t nrows, int seg_len, const float* __restrict__ w, float eps,
                       const float* __restrict__ scale, const float* __restrict__ shift, float rscale, int add_input,
                       T* out) {
  constexpr int NP = C / 256, E = C / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float wv[NP][8];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int e = 0; e < 8; ++e) wv[p][e] = w ? __ldg(w + p * 256 + lane * 8 + e) : 1.f;
  // the warp's next row is loaded before the current one is stored (rows are
  // disjoint, so this is safe when out aliases x)
  const int64_t stride = (int64_t)gridDim.x * 8, first = (int64_t)blockIdx.x * 8 + warp;
  Vec8<T> cur[NP], nxt[NP];
  auto load_row = [&](int64_t row, Vec8<T> (&dst)[NP]) {
    const T* xr = x + row * C;
#pragma unroll
    for (int p = 0; p < NP; ++p) dst[p] = ld_vec8(xr + p * 256 + lane * 8);
  };
  constexpr bool PF = NP <= 2;  // two rows in registers only for C = 512
  if (PF && first < nrows) load_row(first, cur);
  for (int64_t row = first; row < nrows; row += stride) {
    if (!PF) load_row(row, cur);
    else if (row + stride < nrows) load_row(row + stride, nxt);
    float v[NP][8];
    float s = 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      unpack_vec8(cur[p], v[p]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[p][e], v[p][e], s);
    }
    if (PF) {
#pragma unroll
      for (int p = 0; p < NP; ++p) cur[p] = nxt[p];
    }
    s = warp_sum(s);
    const float r = w ? rsqrtf(s / (float)C + eps) : 1.0f;
    const int64_t seg = row / seg_len;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int b = (p * 256 + lane * 8) >> 5;  // the lane's 8 channels lie in one 32-wide block
      const float sc = __ldg(scale + seg * E + b), sh = __ldg(shift + seg * E + b) * 0.1f;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xn = w ? v[p][e] * r * wv[p][e] : v[p][e];
        const float xm = xn * sc + sh;
        const float xo = xn + rscale * (xm - xn);
        o[e] = add_input ? v[p][e] + xo : xo;
      }
      store8(out + row * C + p * 256 + lane * 8, o);
    }
  }
}

// Second MLP layer for SPB segments whose hidden activations hid [SPB][C/4]
// are in shared memory: m = g2 W2q h, scale = 1 + clamp(scale_temp) tanh(m[:E]),
// shift = m[E:] (all 256 threads; sums in byte order of the packed rows).
template <int SPB>
__device__ __forceinline__ void chmod_layer2(const float* hid, int ns, int seg0, int C,
                                             const uint8_t* __restrict__ w2, float g2,
                                             const float* __restrict__ scale_temp, float* __restrict__ scale,
                                             float* __restrict__ shift) {
  const int HIDN = C / 4, E = C / 32;
  const float st = fminf(fmaxf(__ldg(scale_temp), 0.1f), 0.5f);
  const int kb2 = HIDN / 4;
  for (int r = threadIdx.x; r < 2 * E; r += 256) {
    const uint8_t* row = w2 + (size_t)r * kb2;
    float acc[SPB];
#pragma unroll
    for (int z = 0; z < SPB; ++z) acc[z] = 0.f;
#pragma unroll 8
    for (int b = 0; b < kb2; ++b) {
      const uint32_t byte = __ldg(row + b);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float w = tern_val(byte, q);
#pragma unroll
        for (int z = 0; z < SPB; ++z) acc[z] = fmaf(w, hid[z * HIDN + 4 * b + q], acc[z]);
      }
    }
#pragma unroll
    for (int z = 0; z < SPB; ++z) {
      if (z >= ns) break;
      const float a = acc[z] * g2;
      const size_t seg = (size_t)(seg0 + z);
      if (r < E) scale[seg * E + r] = 1.0f + st * tanhf(a);
      else shift[seg * E + (r - E)] = a;
    }
  }
}

// SPB segments per CTA: the packed weights are read once per CTA and every
// weight is applied to SPB segments' activations (register-blocked); each
// segment's sums keep the single-segment order, so results do not depend
// on SPB.
template <int SPB>
__global__ void __launch_bounds__(256)
chmod_mlp_kernel(const float* __restrict__ partial, int nseg, int nch, int seg_len, int C,
                 const uint8_t* __restrict__ w1, const uint8_t* __restrict__ w2, const float* __restrict__ gammas,
                 const float* __restrict__ scale_temp, float* __restrict__ scale, float* __restrict__ shift) {
  extern __shared__ float4 smem4[];
  float* bulk = reinterpret_cast<float*>(smem4);  // [SPB][C]
  float* hid = bulk + SPB * C;                     // [SPB][C/4]
  const int seg0 = blockIdx.x * SPB;
  const int ns = min(SPB, nseg - seg0);
  const int HIDN = C / 4, E = C / 32;
  for (int i = threadIdx.x; i < SPB * C; i += 256) {
    const int j = i / C, c = i - j * C;
    float sum = 0.f;
    if (j < ns)
      for (int k = 0; k < nch; ++k) sum += partial[((size_t)(seg0 + j) * nch + k) * C + c];
    bulk[i] = sum / (float)seg_len;
  }
  __syncthreads();
  const float g1 = __ldg(gammas + 0), g2 = __ldg(gammas + 1);
  const int kb1 = C / 4;
  // rows of kb1 = C/4 bytes are read 16 bytes at a time (C % 64 == 0), several
  // loads in flight; the per-segment accumulation order is byte by byte as before
  const bool vec1 = (kb1 & 15) == 0 && (((uintptr_t)w1) & 15u) == 0;
  for (int j = threadIdx.x; j < HIDN; j += 256) {
    const uint8_t* row = w1 + (size_t)j * kb1;
    float acc[SPB];
#pragma unroll
    for (int z = 0; z < SPB; ++z) acc[z] = 0.f;
    if (vec1) {
#pragma unroll 4
      for (int b16 = 0; b16 < kb1; b16 += 16) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(row + b16));
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) {
            const uint32_t byte = (words[wi] >> (8 * bb)) & 0xffu;
            const int b = b16 + 4 * wi + bb;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float w = tern_val(byte, q);
#pragma unroll
              for (int z = 0; z < SPB; ++z) acc[z] = fmaf(w, bulk[z * C + 4 * b + q], acc[z]);
            }
          }
      }
    } else {
      for (int b = 0; b < kb1; ++b) {
        const uint32_t byte = __ldg(row + b);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float w = tern_val(byte, q);
#pragma unroll
          for (int z = 0; z < SPB; ++z) acc[z] = fmaf(w, bulk[z * C + 4 * b + q], acc[z]);
        }
      }
    }
#pragma unroll
    for (int z = 0; z < SPB; ++z) {
      const float a = acc[z] * g1;
      hid[z * HIDN + j] = a / (1.0f + expf(-a));
    }
  }
  __syncthreads();
  chmod_layer2<SPB>(hid, ns, seg0, C, w2, g2, scale_temp, scale, shift);
}

// Tensor-core form of the MLP's first layer for large segment counts
// (batched decode: one segment per stream row).  The fp32 segment means are
// split into three bf16 rows (hi, mid, lo: hi + mid + lo = bulk to fp32
// precision, with bf16's exponent range), all 3 nseg rows go through one
// GEMM against W1 as dense bf16 (ternary values are exact), and layer 2 sums
// the three fp32 results before the SiLU.
int gemm_bf16_f32out(const __nv_bfloat16* a, int64_t M, int K, const __nv_bfloat16* w, int64_t N, float* y,
                     cudaStream_t s);  // octonion.cu

__global__ void chmod_bulk_split_kernel(const float* __restrict__ partial, int nseg, int nch, int seg_len, int C,
                                        __nv_bfloat16* __restrict__ a) {
  const int64_t total = (int64_t)nseg * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t seg = i / C;
    const int c = (int)(i - seg * C);
    float sum = 0.f;
    for (int k = 0; k < nch; ++k) sum += partial[((size_t)seg * nch + k) * C + c];
    const float b = sum / (float)seg_len;
    const __nv_bfloat16 hi = __float2bfloat16_rn(b);
    const float r1 = b - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    a[i] = hi;
    a[total + i] = mid;
    a[2 * total + i] = lo;
  }
}

template <int SPB>
__global__ void __launch_bounds__(256)
chmod_mlp2_kernel(const float* __restrict__ h1, int nseg, int C, const uint8_t* __restrict__ w2,
                  const float* __restrict__ gammas, const float* __restrict__ scale_temp, float* __restrict__ scale,
                  float* __restrict__ shift) {
  extern __shared__ float4 smem4[];
  float* hid = reinterpret_cast<float*>(smem4);  // [SPB][C/4]
  const int seg0 = blockIdx.x * SPB;
  const int ns = min(SPB, nseg - seg0);
  const int HIDN = C / 4;
  const float g1 = __ldg(gammas + 0), g2 = __ldg(gammas + 1);
  const size_t plane = (size_t)nseg * HIDN;
  for (int i = threadIdx.x; i < SPB * HIDN; i += 256) {
    const int z = i / HIDN, j = i - z * HIDN;
    float v = 0.f;
    if (z < ns) {
      const size_t o = (size_t)(seg0 + z) * HIDN + j;
      v = (h1[o] + h1[plane + o]) + h1[2 * plane + o];
    }
    const float a = v * g1;
    hid[i] = a / (1.0f + expf(-a));
  }
  __syncthreads();
  chmod_layer2<SPB>(hid, ns, seg0, C, w2, g2, scale_temp, scale, shift);
}

// Warp per row.
template <typename T>
__global__ void __launch_bounds__(256)
chmod_apply_kernel(const T* x, int64_t nrows, int C, int seg_len, const float* __restrict__ w, float eps,
                   const float* __restrict__ scale, const float* __restrict__ shift, float rscale, int add_input,
                   T* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = C / 32;
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < nrows; row += (int64_t)gridDim.x * 8) {
    const T* xr = x + row * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = to_f(xr[c]);
      s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    const float r = w ? rsqrtf(s / (float)C + eps) : 1.0f;
    const int64_t seg = row / seg_len;
    const float* sc = scale + seg * E;
    const float* sh = shift + seg * E;
    T* orow = out + row * C;
    for (int c = lane; c < C; c += 32) {
      const float xv = to_f(xr[c]);
      const float xn = w ? xv * r * __ldg(w + c) : xv;
      const int b = c >> 5;
      const float xm = xn * __ldg(sc + b) + __ldg(sh + b) * 0.1f;
      const float xo = xn + rscale * (xm - xn);
      orow[c] = from_f<T>(add_input ? xv + xo : xo);
    }
  }
}

// ---------------------------------------------------------------------------
// Single-row segments (batched decode: each row of the [B*n, 1, C] view is
// its own segment), C = 512, in one kernel instead of stats / bulk split /
// layer-1 GEMM / layer 2 / apply.  A CTA of 256 threads takes 8 rows:
//   rows     warps 0-7, one row each, held in registers for the last step:
//            RMS factor, xn = x r w_norm, which is also the segment mean,
//            split into bf16 hi + mid + lo (their sum is xn to float32
//            precision) as rows z, 8 + z, 16 + z of a 32-row MMA operand
//            (rows 24-31 read one zero row);
//   layer 1  warp w: hidden units 16 w .. 16 w + 15 as m16n8k16 bf16 MMAs
//            over the two 16-row tiles, A the split rows (ldmatrix), B the
//            ternary W1 values decoded from the packed rows staged in shared
//            memory (132-byte rows: the eight rows a warp reads fall in
//            distinct banks); h = SiLU(g1 ((hi + mid) + lo)), the sums of the
//            tensor-core form;
//   layer 2  thread (r, slice) takes 16 hidden units of output r, summed
//            over the 8 slices by shuffles: m = g2 W2q h,
//            scale = 1 + clamp(temp, 0.1, 0.5) tanh(m[:E]), shift = m[E:];
//   apply    out = x + xn + rs (xn scale + 0.1 shift - xn) from the kept rows.
// ---------------------------------------------------------------------------
namespace chrow {
constexpr int C = 512, R = 8, HID = C / 4, E = C / 32, NT = 256;
constexpr int WWORDS = C / 16;          // packed W1 row: 32 words of 16 codes
constexpr int WPITCH = WWORDS + 1;      // shared-memory row pitch in words
constexpr int APITCH = C + 8;           // MMA operand row pitch in bf16 (1040 bytes)
}  // namespace chrow

// bf16 pair (c_lo - 1, c_hi - 1) of two 2-bit codes: the integers 128 + c in
// bf16 less 129 (exact)
__device__ __forceinline__ uint32_t chrow_code_pair(uint32_t c_lo, uint32_t c_hi) {
  const uint32_t v = c_lo | (c_hi << 16) | 0x43004300u;
  __nv_bfloat162 h;
  memcpy(&h, &v, 4);
  h = __hsub2(h, __float2bfloat162_rn(129.0f));
  uint32_t o;
  memcpy(&o, &h, 4);
  return o;
}

template <typename T>
__global__ void __launch_bounds__(chrow::NT)
chmod_rows_kernel(const T* x, int64_t nrows, const float* __restrict__ norm_w, float eps,
                  const uint8_t* __restrict__ w1, const uint8_t* __restrict__ w2, const float* __restrict__ gammas,
                  const float* __restrict__ scale_temp, float rscale, int add_input, float* __restrict__ scale,
                  float* __restrict__ shift, T* out) {
  using namespace chrow;
  __shared__ uint32_t w1s[HID * WPITCH];
  __shared__ __align__(16) __nv_bfloat16 as[25 * APITCH];  // rows z, 8 + z, 16 + z: hi, mid, lo; row 24 zero
  __shared__ float hid[R * HID];
  __shared__ float mod[R * 2 * E];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, t4 = lane & 3;
  const int64_t row0 = (int64_t)blockIdx.x * R;
  // packed W1 (16 KB): all four 16-byte loads of a thread in flight at once
  {
    constexpr int NV = HID * WWORDS / 4 / NT;  // 4
    uint4 wv[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) wv[k] = __ldg(reinterpret_cast<const uint4*>(w1) + tid + k * NT);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i4 = tid + k * NT, r = i4 / (WWORDS / 4), w0 = (i4 % (WWORDS / 4)) * 4;
      uint32_t* d = w1s + r * WPITCH + w0;
      d[0] = wv[k].x;
      d[1] = wv[k].y;
      d[2] = wv[k].z;
      d[3] = wv[k].w;
    }
  }
  // ---- rows
  const int64_t row = row0 + warp;
  const bool has = warp < R && row < nrows;
  float v[2][8];
  float rf = 1.f;
  if (warp < R) {
    float s = 0.f;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      if (has) unpack_vec8(ld_vec8(x + row * C + p * 256 + lane * 8), v[p]);
      else
#pragma unroll
        for (int e = 0; e < 8; ++e) v[p][e] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[p][e], v[p][e], s);
    }
    s = warp_sum(s);
    rf = norm_w ? rsqrtf(s / (float)C + eps) : 1.0f;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint32_t hw[4], mw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float hi2[2], md2[2], lo2[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int c = p * 256 + lane * 8 + e + k;
          const float b = norm_w ? v[p][e + k] * rf * __ldg(norm_w + c) : v[p][e + k];
          const float h = __bfloat162float(__float2bfloat16_rn(b));
          const float r1 = b - h;
          const float m = __bfloat162float(__float2bfloat16_rn(r1));
          hi2[k] = h;
          md2[k] = m;
          lo2[k] = r1 - m;
        }
        hw[e / 2] = pack_bf16(hi2[0], hi2[1]);
        mw[e / 2] = pack_bf16(md2[0], md2[1]);
        lw[e / 2] = pack_bf16(lo2[0], lo2[1]);
      }
      const int c0 = p * 256 + lane * 8;
      *reinterpret_cast<uint4*>(as + warp * APITCH + c0) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(as + (8 + warp) * APITCH + c0) = make_uint4(mw[0], mw[1], mw[2], mw[3]);
      *reinterpret_cast<uint4*>(as + (16 + warp) * APITCH + c0) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  if (tid < APITCH / 8) *reinterpret_cast<uint4*>(as + 24 * APITCH + tid * 8) = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  // ---- layer 1 on the tensor cores: warp w, hidden units 16 w + 8 nt + (0..7)
  const float g1 = __ldg(gammas + 0), g2 = __ldg(gammas + 1);
  {
    // acc[m][nt]: row tile m (rows 16 m ..), hidden n-tile nt; each decoded B
    // fragment serves both row tiles
    float acc[2][2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) acc[m][nt][0] = acc[m][nt][1] = acc[m][nt][2] = acc[m][nt][3] = 0.f;
    const uint32_t abase = (uint32_t)__cvta_generic_to_shared(as);
    const int sh_a = 8 * (t4 >> 1) + 6 - 4 * (t4 & 1);  // code of channel 16 ks + 2 t4 in its word
#pragma unroll 4
    for (int ks = 0; ks < WWORDS; ++ks) {
      uint32_t a[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int arow = min(16 * m + (lane & 15), 24);  // tile 1 rows 8-15 read the zero row
        const uint32_t addr = abase + (uint32_t)((arow * APITCH + ks * 16 + (lane >> 4) * 8) * 2);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(a[m][0]), "=r"(a[m][1]), "=r"(a[m][2]), "=r"(a[m][3])
                     : "r"(addr));
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t wd = w1s[(16 * warp + 8 * nt + gid) * WPITCH + ks];
        // channels 16 ks + 2 t4, +1 (b0) and + 8, + 9 (b1): bytes t4/2 and t4/2 + 2
        const uint32_t b0 = chrow_code_pair((wd >> sh_a) & 3u, (wd >> (sh_a - 2)) & 3u);
        const uint32_t b1 = chrow_code_pair((wd >> (sh_a + 16)) & 3u, (wd >> (sh_a + 14)) & 3u);
        mma16<__nv_bfloat16>(acc[0][nt], a[0], b0, b1);
        mma16<__nv_bfloat16>(acc[1][nt], a[1], b0, b1);
      }
    }
    // row z = gid: hi in tile 0 row gid, mid in tile 0 row gid + 8, lo in tile 1 row gid
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float a1 = ((acc[0][nt][e] + acc[0][nt][2 + e]) + acc[1][nt][e]) * g1;
        hid[gid * HID + 16 * warp + 8 * nt + 2 * t4 + e] = a1 / (1.0f + expf(-a1));
      }
  }
  __syncthreads();
  // ---- layer 2
  {
    const int r = tid >> 3, sl = tid & 7;
    const uint32_t word = __ldg(reinterpret_cast<const uint32_t*>(w2 + (size_t)r * (HID / 4)) + sl);
    float acc[R];
#pragma unroll
    for (int z = 0; z < R; ++z) acc[z] = 0.f;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const float w = (float)((int)((word >> (8 * (q >> 2) + 6 - 2 * (q & 3))) & 3u) - 1);
#pragma unroll
      for (int z = 0; z < R; ++z) acc[z] = fmaf(w, hid[z * HID + 16 * sl + q], acc[z]);
    }
#pragma unroll
    for (int z = 0; z < R; ++z) {
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) acc[z] += __shfl_xor_sync(0xffffffffu, acc[z], o);
      if (sl == 0) mod[z * 2 * E + r] = acc[z] * g2;
    }
  }
  __syncthreads();
  const float st = fminf(fmaxf(__ldg(scale_temp), 0.1f), 0.5f);
  if (tid < R * 2 * E) {
    const int z = tid / (2 * E), k = tid % (2 * E);
    if (row0 + z < nrows) {
      const float a = mod[tid];
      if (k < E) scale[(row0 + z) * E + k] = 1.0f + st * tanhf(a);
      else shift[(row0 + z) * E + (k - E)] = a;
    }
  }
  // ---- apply (each thread recomputes its block's scale from the same m)
  if (has) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int b = (p * 256 + lane * 8) >> 5;
      const float sc = 1.0f + st * tanhf(mod[warp * 2 * E + b]), sh = mod[warp * 2 * E + E + b] * 0.1f;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = p * 256 + lane * 8 + e;
        const float xn = norm_w ? v[p][e] * rf * __ldg(norm_w + c) : v[p][e];
        const float xm = xn * sc + sh;
        const float xo = xn + rscale * (xm - xn);
        o[e] = add_input ? v[p][e] + xo : xo;
      }
      store8(out + row * C + p * 256 + lane * 8, o);
    }
  }
}

}  // namespace walsh

using namespace walsh;

extern "C" int walsh_chmod_chunk_rows(int seg_len) {
  (void)seg_len;
  return kChunkRows;
}

extern "C" walsh_status walsh_chmod_stats(const void* x, int dtype, int64_t nrows, int C, int seg_len,
                                          const float* norm_w, float norm_eps, float* partial, void* stream) {
  if (int e = injected("chmod_stats")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(x && partial);
  WALSH_CHECK_SHAPE(nrows > 0 && C > 0 && C % 32 == 0 && seg_len > 0 && nrows % seg_len == 0);
  const int64_t nseg = nrows / seg_len;
  WALSH_CHECK_SHAPE(nseg <= 65535);
  dim3 grid((seg_len + kChunkRows - 1) / kChunkRows, (unsigned)nseg);
  cudaStream_t s = (cudaStream_t)stream;
  if (C == 512 && (((uintptr_t)x) & 15u) == 0)
    return WALSH_DISPATCH_DTYPE(dtype, T, (chmod_stats_vec_kernel<T, 512><<<grid, 256, 0, s>>>(
                                               (const T*)x, seg_len, norm_w, norm_eps, partial),
                                           launch_status()));
  return WALSH_DISPATCH_DTYPE(dtype, T, (chmod_stats_kernel<T><<<grid, 256, 0, s>>>((const T*)x, C, seg_len, norm_w,
                                                                                  norm_eps, partial),
                                         launch_status()));
}

extern "C" walsh_status walsh_chmod_mlp(const float* partial, int nseg, int seg_len, int C, const uint8_t* w1_2bit,
                                        const uint8_t* w2_2bit, const float* gammas, const float* scale_temp,
                                        float* scale, float* shift, void* stream) {
  if (int e = injected("chmod_mlp")) return e;
  WALSH_CHECK_ARG(partial && w1_2bit && w2_2bit && gammas && scale_temp && scale && shift);
  WALSH_CHECK_SHAPE(nseg > 0 && seg_len > 0 && C > 0 && C % 32 == 0);
  const int nch = (seg_len + kChunkRows - 1) / kChunkRows;
  cudaStream_t s = (cudaStream_t)stream;
  // segments per CTA: enough CTAs to fill the SMs, weights shared beyond that
  const int spb = nseg >= 148 * 8 ? 8 : nseg >= 148 * 4 ? 4 : nseg >= 148 * 2 ? 2 : 1;
  const size_t smem = (size_t)spb * (C + C / 4) * sizeof(float);
  const unsigned grid = (unsigned)((nseg + spb - 1) / spb);
  auto go = [&](auto kernel) -> int {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return launch_status();
    kernel<<<grid, 256, smem, s>>>(partial, nseg, nch, seg_len, C, w1_2bit, w2_2bit, gammas, scale_temp, scale,
                                   shift);
    return launch_status();
  };
  if (smem > 200 * 1024) return WALSH_ERR_SHAPE;
  switch (spb) {
    case 8: return go(chmod_mlp_kernel<8>);
    case 4: return go(chmod_mlp_kernel<4>);
    case 2: return go(chmod_mlp_kernel<2>);
    default: return go(chmod_mlp_kernel<1>);
  }
}

extern "C" int64_t walsh_chmod_mlp_tc_scratch_bytes(int nseg, int C) {
  return ((int64_t)3 * nseg * C * 2 + 255) / 256 * 256 + (int64_t)3 * nseg * (C / 4) * 4;
}

extern "C" walsh_status walsh_chmod_mlp_tc(const float* partial, int nseg, int seg_len, int C, const void* w1_bf16,
                                           const uint8_t* w2_2bit, const float* gammas, const float* scale_temp,
                                           void* scratch, float* scale, float* shift, void* stream) {
  if (int e = injected("chmod_mlp_tc")) return e;
  WALSH_CHECK_ARG(partial && w1_bf16 && w2_2bit && gammas && scale_temp && scratch && scale && shift);
  WALSH_CHECK_SHAPE(nseg > 0 && seg_len > 0 && C > 0 && C % 64 == 0 && C <= 8192 &&
                    (int64_t)3 * nseg <= 2147483647LL);
  if ((((uintptr_t)w1_bf16) | ((uintptr_t)scratch)) & 15u) return WALSH_ERR_ALIGN;
  const int nch = (seg_len + kChunkRows - 1) / kChunkRows;
  cudaStream_t s = (cudaStream_t)stream;
  __nv_bfloat16* a = reinterpret_cast<__nv_bfloat16*>(scratch);
  float* h1 = reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) +
                                       ((int64_t)3 * nseg * C * 2 + 255) / 256 * 256);
  const int64_t total = (int64_t)nseg * C;
  const unsigned sgrid = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
  chmod_bulk_split_kernel<<<sgrid, 256, 0, s>>>(partial, nseg, nch, seg_len, C, a);
  if (int e = launch_status()) return e;
  if (int e = gemm_bf16_f32out(a, (int64_t)3 * nseg, C, reinterpret_cast<const __nv_bfloat16*>(w1_bf16), C / 4,
                               h1, s))
    return e;
  const int spb = nseg >= 148 * 8 ? 8 : nseg >= 148 * 4 ? 4 : nseg >= 148 * 2 ? 2 : 1;
  const size_t smem = (size_t)spb * (C / 4) * sizeof(float);
  const unsigned grid = (unsigned)((nseg + spb - 1) / spb);
  auto go = [&](auto kernel) -> int {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return launch_status();
    kernel<<<grid, 256, smem, s>>>(h1, nseg, C, w2_2bit, gammas, scale_temp, scale, shift);
    return launch_status();
  };
  switch (spb) {
    case 8: return go(chmod_mlp2_kernel<8>);
    case 4: return go(chmod_mlp2_kernel<4>);
    case 2: return go(chmod_mlp2_kernel<2>);
    default: return go(chmod_mlp2_kernel<1>);
  }
}

extern "C" walsh_status walsh_chmod_apply(const void* x, int dtype, int64_t nrows, int C, int seg_len,
                                          const float* norm_w, float norm_eps, const float* scale, const float* shift,
                                          float residual_scale, int add_input, void* out, void* stream) {
  if (int e = injected("chmod_apply")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(x && scale && shift && out);
  WALSH_CHECK_SHAPE(nrows > 0 && C > 0 && C % 32 == 0 && seg_len > 0 && nrows % seg_len == 0);
  int64_t g = (nrows + 7) / 8;
  if (g > 148 * 32) g = 148 * 32;
  cudaStream_t s = (cudaStream_t)stream;
  if (C % 256 == 0 && C <= 2048 && ((((uintptr_t)x) | ((uintptr_t)out)) & 15u) == 0) {
    if (C == 512)
      return WALSH_DISPATCH_DTYPE(dtype, T, (chmod_apply_vec_kernel<T, 512><<<(unsigned)g, 256, 0, s>>>(
                                                 (const T*)x, nrows, seg_len, norm_w, norm_eps, scale, shift,
                                                 residual_scale, add_input, (T*)out),
                                             launch_status()));
    if (C == 2048)
      return WALSH_DISPATCH_DTYPE(dtype, T, (chmod_apply_vec_kernel<T, 2048><<<(unsigned)g, 256, 0, s>>>(
                                                 (const T*)x, nrows, seg_len, norm_w, norm_eps, scale, shift,
                                                 residual_scale, add_input, (T*)out),
                                             launch_status()));
  }
  return WALSH_DISPATCH_DTYPE(dtype, T, (chmod_apply_kernel<T><<<(unsigned)g, 256, 0, s>>>(
                                             (const T*)x, nrows, C, seg_len, norm_w, norm_eps, scale, shift,
                                             residual_scale, add_input, (T*)out),
                                         launch_status()));
}

extern "C" walsh_status walsh_chmod_rows_fwd(const void* x, int dtype, int64_t nrows, int C, const float* norm_w,
                                             float norm_eps, const uint8_t* w1_2bit, const uint8_t* w2_2bit,
                                             const float* gammas, const float* scale_temp, float residual_scale,
                                             int add_input, float* scale, float* shift, void* out, void* stream) {
  if (int e = injected("chmod_rows_fwd")) return e;
  WALSH_CHECK_ARG(x && w1_2bit && w2_2bit && gammas && scale_temp && scale && shift && out);
  WALSH_CHECK_SHAPE(nrows > 0 && C == chrow::C);
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  if ((((uintptr_t)x) | ((uintptr_t)out) | ((uintptr_t)w1_2bit)) & 15u || ((uintptr_t)w2_2bit) & 3u)
    return WALSH_ERR_ALIGN;
  const int64_t grid = (nrows + chrow::R - 1) / chrow::R;
  if (grid > 2147483647LL) return WALSH_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == WALSH_BF16)
    chmod_rows_kernel<__nv_bfloat16><<<(unsigned)grid, chrow::NT, 0, s>>>(
        (const __nv_bfloat16*)x, nrows, norm_w, norm_eps, w1_2bit, w2_2bit, gammas, scale_temp, residual_scale,
        add_input, scale, shift, (__nv_bfloat16*)out);
  else
    chmod_rows_kernel<__half><<<(unsigned)grid, chrow::NT, 0, s>>>(
        (const __half*)x, nrows, norm_w, norm_eps, w1_2bit, w2_2bit, gammas, scale_temp, residual_scale, add_input,
        scale, shift, (__half*)out);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free channel modulation.
//
// walsh_chmod_stats / _mlp / _apply leave the scratch (per-chunk partial
// sums, per-segment scale and shift) to the caller.  Some callers cannot
// obtain device memory at the moment they run the layer: a host whose device
// memory is planned once at start-up and which has no allocator at call time
// (a plain C runtime, a memory-budgeted serving process), or code running
// where an allocation would have to synchronise the device.  For them the
// entry point below keeps the scratch in a fixed array in the library's own
// device memory; the call itself allocates nothing.
//
// Every scratch word a step reads was written earlier in the same call
// (stats writes every partial, mlp every scale and shift), so nothing has to
// start at zero.  The array is one per device and shared by all callers:
// two calls whose executions overlap on the device (other streams, other
// host threads) race on it and must be ordered by the caller.
// ---------------------------------------------------------------------------

namespace walsh {

constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 20;  // 4 MiB of float32
constexpr int64_t kNoAllocAlignFloats = 64;                  // 256-byte sub-buffers
constexpr int kNoAllocMaxContexts = 64;

__device__ __align__(256) float g_chmod_scratch[kNoAllocScratchFloats];

ContextAddressCache<kNoAllocMaxContexts> g_chmod_scratch_cache;

static int64_t round_up_floats(int64_t n) { return (n + kNoAllocAlignFloats - 1) / kNoAllocAlignFloats * kNoAllocAlignFloats; }

// Driver calls reached through the runtime's entry-point table (no link
// against libcuda): the current context and its process-unique id.
using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);

static bool ctx_fns(PfnCtxGetCurrent* get_cur, PfnCtxGetId* get_id) {
  static PfnCtxGetCurrent cur = nullptr;
  static PfnCtxGetId id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      cur = reinterpret_cast<PfnCtxGetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      id = reinterpret_cast<PfnCtxGetId>(p);
    cudaGetLastError();
  });
  *get_cur = cur;
  *get_id = id;
  return cur && id;
}

// Id of the context current on this thread, 0 when there is none.
static uint64_t current_ctx_id(PfnCtxGetCurrent get_cur, PfnCtxGetId get_id) {
  CUcontext ctx = nullptr;
  if (get_cur(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch array in the current context.  The set-up
// (cudaGetSymbolAddress, with the caller's device current) runs on the first
// call in each context and is cached under the context's id; a device reset or
// a different current context on the same device is a new context and is
// looked up again.  Every later call costs two driver queries.
static walsh_status chmod_scratch_for_current_context(float** out) {
  PfnCtxGetCurrent get_cur;
  PfnCtxGetId get_id;
  if (!ctx_fns(&get_cur, &get_id)) return WALSH_ERR_NOT_INIT;
  uint64_t id = current_ctx_id(get_cur, get_id);
  if (void* p = g_chmod_scratch_cache.find(id)) {
    *out = static_cast<float*>(p);
    return WALSH_OK;
  }
  // set-up: the lookup also makes the device's primary context current when
  // no context was yet
  void* addr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&addr, g_chmod_scratch);
  if (e != cudaSuccess || addr == nullptr) {
    cudaGetLastError();
    return WALSH_ERR_NOT_INIT;
  }
  id = current_ctx_id(get_cur, get_id);
  if (id == 0) return WALSH_ERR_NOT_INIT;
  g_chmod_scratch_cache.insert(id, addr);
  *out = static_cast<float*>(addr);
  return WALSH_OK;
}

}  // namespace walsh

// Floats of scratch a call needs: partial [nseg, nchunk, C], scale and shift
// [nseg, C/32], each sub-buffer rounded up to 256 bytes.
static int64_t chmod_noalloc_scratch_floats(int64_t nseg, int C, int seg_len) {
  const int64_t nch = (seg_len + kChunkRows - 1) / kChunkRows;
  const int64_t E = C / 32;
  return round_up_floats(nseg * nch * C) + 2 * round_up_floats(nseg * E);
}

extern "C" walsh_status walsh_chmod_fwd_noalloc(const void* x, int dtype, int64_t nrows, int C, int seg_len,
                                                const float* norm_w, float norm_eps, const uint8_t* w1_2bit,
                                                const uint8_t* w2_2bit, const float* gammas,
                                                const float* scale_temp, float residual_scale, int add_input,
                                                void* out, void* stream) {
  if (int e = injected("chmod_fwd_noalloc")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(x && w1_2bit && w2_2bit && gammas && scale_temp && out);
  WALSH_CHECK_SHAPE(nrows > 0 && C > 0 && C % 32 == 0 && seg_len > 0 && nrows % seg_len == 0);
  const int64_t nseg = nrows / seg_len;
  WALSH_CHECK_SHAPE(nseg <= 65535);
  if (chmod_noalloc_scratch_floats(nseg, C, seg_len) > kNoAllocScratchFloats) return WALSH_ERR_SCRATCH;
  float* scratch = nullptr;
  if (walsh_status st = chmod_scratch_for_current_context(&scratch)) return st;
  const int64_t nch = (seg_len + kChunkRows - 1) / kChunkRows;
  float* partial = scratch;
  float* scale = partial + round_up_floats(nseg * nch * C);
  float* shift = scale + round_up_floats(nseg * (C / 32));
  if (walsh_status st = walsh_chmod_stats(x, dtype, nrows, C, seg_len, norm_w, norm_eps, partial, stream)) return st;
  if (walsh_status st = walsh_chmod_mlp(partial, (int)nseg, seg_len, C, w1_2bit, w2_2bit, gammas, scale_temp, scale,
                                        shift, stream))
    return st;
  return walsh_chmod_apply(x, dtype, nrows, C, seg_len, norm_w, norm_eps, scale, shift, residual_scale, add_input,
                           out, stream);
}
