// Octonion (Cayley-Dickson) layers as tensor-core GEMMs with fused epilogues.
//
// Reference: OctonionTernaryLinearRef / OctonionFusedLinear
// (src/model/physics.py:53-82, src/model/cayley_dickson_cuda.py:622-668):
//   y_i = beta * sum_j SIGN[i][j] x_j @ Wq[WIDX[i][j]]^T   (i, j = 0..7 parts)
// with Wq the unscaled absmean ternary of the [8, out_o, in_o] latent.  The
// host expands the eight blocks once per parameter version into the dense
// signed matrix W[(i, o), (j, k)] = SIGN[i][j] Wq[WIDX[i][j]][o][k] (ternary,
// exact in fp16/bf16), so every octonion layer is one GEMM y = x W^T whose
// epilogue applies beta per output column and the op that follows:
//   plain   y = beta . (x W^T)                                (module forward)
//   qkv     q/k/v of CausalSelfAttention in one GEMM (N = 3C): beta, RoPE
//           on the interleaved pairs, q written [B, H, T, hd], k/v written
//           into the caches at rows start_pos..           (chassis.py:424-447)
//   swiglu  gate and up rows interleaved (N = 2 hidden): h = silu(g) * u
//                                                            (chassis.py:497-507)
//   post    the mHC site epilogue x'_i = sum_j H_res[i][j] x_j + H_post[i] f
//           (wo with the octonion head mixer folded in, and down_proj)
//                                                            (mhc.py:345-381)
//
// Mainloop: CTA tile 128 x 128, 8 warps of 64 x 32, K staged 32 wide through a
// 3-stage cp.async pipeline; mma.sync m16n8k16 with fp32 accumulation.
// Operand types: fp16 x with fp16 W; bf16 x with bf16 W; fp32 x split in
// registers into bf16 hi + lo (x_hi W + x_lo W, and + x_hi W_lo when a W_lo
// correction matrix is given), which keeps float32 accuracy.
#include <cudaTypedefs.h>
#include <math_constants.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "mma.cuh"
#include "tc05.cuh"
#include "tma_host.cuh"

namespace walsh {

// The tcgen05 mainloop is used for 16-bit operands unless switched off with
// walsh_octo_set_mainloop (tests run both mainloops on the same inputs).
static int g_octo_tc05 = 1;
static inline bool octo_tc05_enabled() { return g_octo_tc05 != 0; }

namespace octo {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3, LD = BK + 8, NT = 256;

template <typename TA>
using TE = typename std::conditional<std::is_same<TA, __half>::value, __half, __nv_bfloat16>::type;

template <typename TA>
constexpr int stage_bytes() {
  return BM * LD * (int)sizeof(TA) + 2 * BN * LD * 2;  // A, W_hi, W_lo
}
template <typename TA>
constexpr int smem_bytes() {
  return STAGES * stage_bytes<TA>();
}

__device__ __forceinline__ void split_bf16(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(a, b);
  const float2 h = unpack2<__nv_bfloat16>(hi);
  lo = pack_bf16(a - h.x, b - h.y);
}

template <typename T>
__device__ __forceinline__ void store2(T* p, float a, float b);
template <>
__device__ __forceinline__ void store2<float>(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
template <>
__device__ __forceinline__ void store2<__half>(__half* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = pack_f16_sat(a, b);
}
template <>
__device__ __forceinline__ void store2<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16(a, b);
}

template <typename T>
__device__ __forceinline__ float2 load2(const T* p);
template <>
__device__ __forceinline__ float2 load2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 load2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return unpack2<__nv_bfloat16>(*reinterpret_cast<const uint32_t*>(p));
}
template <>
__device__ __forceinline__ float2 load2<__half>(const __half* p) {
  return unpack2<__half>(*reinterpret_cast<const uint32_t*>(p));
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
  store8(p, v);
  store8(p + 8, v + 8);
}
template <typename T>
__device__ __forceinline__ void load16(const T* p, float* v) {
  load8(p, v);
  load8(p + 8, v + 8);
}

// ---- epilogues: operator() once per (row m, column pair n, n+1), n even;
// chunk16 once per row and 16 consecutive columns n..n+15 (n a multiple of
// 16, destination rows aligned for 16-byte vectors; the launcher checks) ----
template <typename TY>
struct EpiPlain {
  const float* scale;
  TY* y;
  int64_t N;
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float v0, float v1) const {
    store2(y + m * N + n, v0 * __ldg(scale + n), v1 * __ldg(scale + n + 1));
  }
  __device__ __forceinline__ void chunk16(int64_t m, int64_t n, const float* v) const {
    float o[16];
    const float4* s4 = reinterpret_cast<const float4*>(scale + n);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 sv = __ldg(s4 + j);
      o[4 * j] = v[4 * j] * sv.x;
      o[4 * j + 1] = v[4 * j + 1] * sv.y;
      o[4 * j + 2] = v[4 * j + 2] * sv.z;
      o[4 * j + 3] = v[4 * j + 3] * sv.w;
    }
    store16(y + m * N + n, o);
  }
  __device__ __forceinline__ void chunk32(int64_t m, int64_t n, const float* v) const {
    chunk16(m, n, v);
    chunk16(m, n + 16, v + 16);
  }
  // v[j] *= scale[n + j], j < 32 (n a multiple of 32, scale 16-byte aligned)
  __device__ __forceinline__ void scale32(int64_t n, float* v) const {
    const float4* s4 = reinterpret_cast<const float4*>(scale + n);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 sv = __ldg(s4 + j);
      v[4 * j] *= sv.x;
      v[4 * j + 1] *= sv.y;
      v[4 * j + 2] *= sv.z;
      v[4 * j + 3] *= sv.w;
    }
  }
  __host__ bool vec_ok() const { return N % 16 == 0 && (((uintptr_t)scale) & 15u) == 0; }
  // TMA-store form: whole 32-column blocks (scale32), y 16-byte aligned
  __host__ bool tma_ok() const { return vec_ok() && N % 32 == 0 && (((uintptr_t)y) & 15u) == 0; }
  using out_t = TY;
  static constexpr int kWarpScratch = 0;  // has a warp-cooperative path (warp_block)
  static constexpr int kRowEpilogue = 0;  // one call per accumulator row (row)
  static constexpr int kHalfRow = 0;      // one call per row and 128-column half (half_row)
  static constexpr int kTmaStore = 1;     // scale32 + the kernel's TMA-store path
};

template <typename TY>
struct EpiQkv {
  const float* scale;  // [3C]
  TY* q;               // [B, H, T, hd]
  TY* kc;              // [B, H, ctx, hd]
  TY* vc;
  const float* cos;  // [T, hd/2]: rows of the tokens' own positions
  const float* sin;
  int T, n_head, hd, C, ctx, start_pos;
  int c_shift, hd_shift;  // log2 C and log2 hd when they are powers of two, else -1
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float v0, float v1) const {
    const int which = (int)(n / C);
    const int c = (int)(n - (int64_t)which * C);
    const int head = c / hd, d = c - head * hd;
    const int b = (int)(m / T), t = (int)(m - (int64_t)b * T);
    v0 *= __ldg(scale + n);
    v1 *= __ldg(scale + n + 1);
    if (which < 2) {  // the roundings of the pair form in half_row
      const float cs = __ldg(cos + (size_t)t * (hd / 2) + (d >> 1)), sn = __ldg(sin + (size_t)t * (hd / 2) + (d >> 1));
      const float r0 = fmaf(v1, -sn, __fmul_rn(v0, cs)), r1 = fmaf(v0, sn, __fmul_rn(v1, cs));
      v0 = r0;
      v1 = r1;
    }
    TY* dst = which == 0 ? q + (((size_t)b * n_head + head) * T + t) * hd + d
                         : (which == 1 ? kc : vc) + (((size_t)b * n_head + head) * ctx + start_pos + t) * hd + d;
    store2(dst, v0, v1);
  }
  // 16 columns = 16 dims of one head (hd a multiple of 16; the launcher checks
  // M < 2^31 and 16-byte aligned rows of cos / sin / scale, so the index math is
  // 32-bit and the table rows are read as float4)
  __device__ __forceinline__ void chunk16(int64_t m, int64_t n, const float* v) const {
    const int mi = (int)m, ni = (int)n;
    const int which = c_shift >= 0 ? ni >> c_shift : ni / C;
    const int c = ni - which * C;
    const int head = hd_shift >= 0 ? c >> hd_shift : c / hd, d = c - head * hd;
    const int b = mi / T, t = mi - b * T;
    float o[16];
    const float4* s4 = reinterpret_cast<const float4*>(scale + ni);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 sv = __ldg(s4 + j);
      o[4 * j] = v[4 * j] * sv.x;
      o[4 * j + 1] = v[4 * j + 1] * sv.y;
      o[4 * j + 2] = v[4 * j + 2] * sv.z;
      o[4 * j + 3] = v[4 * j + 3] * sv.w;
    }
    if (which < 2) {
      const float4* cr = reinterpret_cast<const float4*>(cos + (size_t)t * (hd / 2) + (d >> 1));
      const float4* sr = reinterpret_cast<const float4*>(sin + (size_t)t * (hd / 2) + (d >> 1));
      const float4 c0 = __ldg(cr), c1 = __ldg(cr + 1), s0 = __ldg(sr), s1 = __ldg(sr + 1);
      const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // the roundings of the pair form in half_row
        const float a = o[2 * j], bb = o[2 * j + 1];
        o[2 * j] = fmaf(bb, -sn[j], __fmul_rn(a, cs[j]));
        o[2 * j + 1] = fmaf(a, sn[j], __fmul_rn(bb, cs[j]));
      }
    }
    TY* dst = which == 0 ? q + (((size_t)b * n_head + head) * T + t) * hd + d
                         : (which == 1 ? kc : vc) + (((size_t)b * n_head + head) * ctx + start_pos + t) * hd + d;
    store16(dst, o);
  }
  __device__ __forceinline__ void chunk32(int64_t m, int64_t n, const float* v) const {
    chunk16(m, n, v);
    chunk16(m, n + 16, v + 16);
  }
  __host__ bool vec_ok() const {
    return hd % 16 == 0 && C % 16 == 0 && ((((uintptr_t)cos) | ((uintptr_t)sin) | ((uintptr_t)scale)) & 15u) == 0;
  }
  static constexpr int kWarpScratch = 0;
  static constexpr int kRowEpilogue = 0;
  // Row path of the tcgen05 kernel for hd = 16: the 3C column scales are
  // staged in shared memory once per CTA, and per tile a thread loads its
  // token's 8 cos and 8 sin values once (every head of the row uses the same
  // 8 frequencies) instead of once per 16 columns, then streams its 128
  // accumulator columns (two 32-column tensor-memory loads in flight).
  static constexpr int kHalfRow = 1;
  static constexpr int kRowScratch = 6144 * 4;  // 3C <= 6144
  __host__ bool half_row_ok() const { return hd == 16 && C % 128 == 0 && 3 * C <= 6144 && vec_ok(); }
  // all 256 epilogue threads (t = 0..255), before the first tile
  __device__ __forceinline__ void stage(float* ws, int t) const {
    for (int i = t; i < 3 * C; i += 256) ws[i] = __ldg(scale + i);
  }
  // columns n0 .. n0 + 127 of row m (one of q | k | v: C % 128 == 0); all 32
  // lanes call it (tensor-memory loads are warp-wide), rows past M store nothing
  __device__ __forceinline__ void half_row(int64_t m, int64_t n0, uint32_t tacc, const float* ws, int64_t M) const {
    const bool valid = m < M;
    const int mi = valid ? (int)m : 0, ni = (int)n0;
    const int b = mi / T, t = mi - b * T;
    const int which = c_shift >= 0 ? ni >> c_shift : ni / C;
    float cs[8], sn[8];
    if (which < 2) {
      const float4* cr = reinterpret_cast<const float4*>(cos + (size_t)t * 8);
      const float4* sr = reinterpret_cast<const float4*>(sin + (size_t)t * 8);
      const float4 c0 = __ldg(cr), c1 = __ldg(cr + 1), s0 = __ldg(sr), s1 = __ldg(sr + 1);
      cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
      sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
    }
    const int head0 = (ni - which * C) >> 4;
    const size_t hstride = (size_t)(which == 0 ? T : ctx) * 16;  // elements between heads
    TY* row = which == 0 ? q + ((size_t)b * n_head * T + t) * 16
                         : (which == 1 ? kc : vc) + ((size_t)b * n_head * ctx + start_pos + t) * 16;
    // RoPE on pairs (a, b) -> (a c - b s, a s + b c) as two f32x2 operations:
    // (b, a) (-s, s) + (a, b) (c, c)
    uint64_t rc[8], rs[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      rc[j] = which < 2 ? f2_dup(cs[j]) : 0;
      rs[j] = which < 2 ? f2_pack(-sn[j], sn[j]) : 0;
    }
#pragma unroll 1
    for (int c = 0; c < 128; c += 64) {
      float v[64];
      tc05::tmem_ld32_nowait(tacc + (uint32_t)c, v);
      tc05::tmem_ld32_nowait(tacc + (uint32_t)c + 32, v + 32);
      tc05::tmem_wait_ld();
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        uint32_t w[8];
        const float4* s4 = reinterpret_cast<const float4*>(ws + ni + c + 16 * hh);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 sv = s4[j];
          const float* vv = v + 16 * hh + 4 * j;
          uint64_t p0 = f2_mul(f2_pack(vv[0], vv[1]), f2_pack(sv.x, sv.y));
          uint64_t p1 = f2_mul(f2_pack(vv[2], vv[3]), f2_pack(sv.z, sv.w));
          if (which < 2) {
            p0 = f2_fma(f2_swap(p0), rs[2 * j], f2_mul(p0, rc[2 * j]));
            p1 = f2_fma(f2_swap(p1), rs[2 * j + 1], f2_mul(p1, rc[2 * j + 1]));
          }
          w[2 * j] = pack2<TY>(f2_lo(p0), f2_hi(p0));
          w[2 * j + 1] = pack2<TY>(f2_lo(p1), f2_hi(p1));
        }
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(row + (size_t)(head0 + (c >> 4) + hh) * hstride);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
  }
};

// fp32 accumulator rows stored unscaled: y [M, N] float; any N (the vector
// path needs N % 16 == 0 and a 16-byte aligned y, else scalar stores)
struct EpiStoreF32 {
  float* y;
  int64_t N;
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float v0, float v1) const {
    y[m * N + n] = v0;
    if (n + 1 < N) y[m * N + n + 1] = v1;
  }
  __device__ __forceinline__ void chunk16(int64_t m, int64_t n, const float* v) const {
    float4* d = reinterpret_cast<float4*>(y + m * N + n);
#pragma unroll
    for (int j = 0; j < 4; ++j) d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  __device__ __forceinline__ void chunk32(int64_t m, int64_t n, const float* v) const {
    chunk16(m, n, v);
    chunk16(m, n + 16, v + 16);
  }
  __host__ bool vec_ok() const { return N % 16 == 0 && (((uintptr_t)y) & 15u) == 0; }
  static constexpr int kWarpScratch = 0, kRowEpilogue = 0, kHalfRow = 0;
};

template <typename TY>
struct EpiSwiglu {
  const float* scale;  // [2 hidden], interleaved like the weight rows
  TY* h;               // [M, hidden]
  int64_t hid;
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float g, float u) const {
    g *= __ldg(scale + n);
    u *= __ldg(scale + n + 1);
    h[m * hid + (n >> 1)] = from_f<TY>(g / (1.0f + expf(-g)) * u);
  }
  __device__ __forceinline__ void chunk16(int64_t m, int64_t n, const float* v) const {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = v[2 * j] * __ldg(scale + n + 2 * j), u = v[2 * j + 1] * __ldg(scale + n + 2 * j + 1);
      o[j] = g / (1.0f + expf(-g)) * u;
    }
    store8(h + m * hid + (n >> 1), o);
  }
  // 16 outputs h[m, n/2 .. n/2 + 15]; fast exp and division (16-bit output)
  __device__ __forceinline__ void chunk32(int64_t m, int64_t n, const float* v) const {
    float o[16];
    const float4* s4 = reinterpret_cast<const float4*>(scale + n);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 sv = __ldg(s4 + j);
      o[2 * j] = siluf_(v[4 * j] * sv.x) * (v[4 * j + 1] * sv.y);
      o[2 * j + 1] = siluf_(v[4 * j + 2] * sv.z) * (v[4 * j + 3] * sv.w);
    }
    store16(h + m * hid + (n >> 1), o);
  }
  __host__ bool vec_ok() const { return hid % 8 == 0 && (((uintptr_t)scale) & 15u) == 0; }
  static constexpr int kWarpScratch = 0;
  static constexpr int kRowEpilogue = 0, kHalfRow = 0;
};

template <typename TX>
struct EpiPost {
  const float* scale;  // [C]
  const TX* x;         // [M, 4, C]  (may alias xo)
  const float* hmix;   // [M, 24]: H_pre | H_post | H_res (row-major 4 x 4)
  TX* xo;
  int C;
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float f0, float f1) const {
    f0 *= __ldg(scale + n);
    f1 *= __ldg(scale + n + 1);
    const float* hm = hmix + m * kMapRows;
    const size_t base = (size_t)m * 4 * C + n;
    const float2 x0 = load2(x + base), x1 = load2(x + base + C), x2 = load2(x + base + 2 * C),
                 x3 = load2(x + base + 3 * C);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float* hr = hm + 8 + 4 * r;
      const float a = (((hr[0] * x0.x + hr[1] * x1.x) + hr[2] * x2.x) + hr[3] * x3.x) + hm[4 + r] * f0;
      const float b = (((hr[0] * x0.y + hr[1] * x1.y) + hr[2] * x2.y) + hr[3] * x3.y) + hm[4 + r] * f1;
      store2(xo + base + (size_t)r * C, a, b);
    }
  }
  __device__ __forceinline__ void chunk16(int64_t m, int64_t n, const float* v) const {
    const float* hm = hmix + m * kMapRows;
    const size_t base = (size_t)m * 4 * C + n;
    float xs[4][16];
#pragma unroll
    for (int j = 0; j < 4; ++j) load16(x + base + (size_t)j * C, xs[j]);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float* hr = hm + 8 + 4 * r;
      const float hp = hm[4 + r];
      float o[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float f = v[e] * __ldg(scale + n + e);
        o[e] = (((hr[0] * xs[0][e] + hr[1] * xs[1][e]) + hr[2] * xs[2][e]) + hr[3] * xs[3][e]) + hp * f;
      }
      store16(xo + base + (size_t)r * C, o);
    }
  }
  // all 4 x 32 stream values are loaded before any store (x and xo may alias)
  __device__ __forceinline__ void chunk32(int64_t m, int64_t n, const float* v) const {
    static_assert(sizeof(TX) == 2 || sizeof(TX) == 4, "stream type");
    const float* hm = hmix + m * kMapRows;
    float hr[16], hp[4];
#pragma unroll
    for (int i = 0; i < 16; ++i) hr[i] = __ldg(hm + 8 + i);
#pragma unroll
    for (int i = 0; i < 4; ++i) hp[i] = __ldg(hm + 4 + i);
    const size_t base = (size_t)m * 4 * C + n;
    if constexpr (sizeof(TX) == 2) {
      uint4 xr[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int k = 0; k < 4; ++k) xr[j][k] = *reinterpret_cast<const uint4*>(x + base + (size_t)j * C + 8 * k);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float xf[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) unpack8(xr[j][k], xf[j], (const TX*)nullptr);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float f = v[8 * k + e] * __ldg(scale + n + 8 * k + e);
            o[e] = (((hr[4 * r] * xf[0][e] + hr[4 * r + 1] * xf[1][e]) + hr[4 * r + 2] * xf[2][e]) +
                    hr[4 * r + 3] * xf[3][e]) + hp[r] * f;
          }
          store8(xo + base + (size_t)r * C + 8 * k, o);
        }
      }
    } else {
      chunk16(m, n, v);
      chunk16(m, n + 16, v + 16);
    }
  }
  __host__ bool vec_ok() const {
    return C % 16 == 0 && ((((uintptr_t)hmix) | ((uintptr_t)scale)) & 15u) == 0;
  }
  // 16-bit streams: a warp's whole 32-row x 128-column block.  Per 32-column
  // chunk the accumulator rows (lane i = row i) are staged through shared
  // memory so that four lanes cover one token row (8 columns each: 16-byte
  // stream accesses, 8 rows per pass); the stream rows and mixing
  // coefficients of the next two passes are already in flight (cp.async into
  // a two-slot ring) while the current pass is mixed.
  static constexpr int kPitch = 36;                      // floats per staged row
  static constexpr int kYBytes = 32 * kPitch * 4;        // staged 32 x 32 chunk
  static constexpr int kXSlot = 8 * 4 * 64;              // 8 rows x 4 streams x 32 columns (16-bit)
  static constexpr int kHSlot = 8 * 80;                  // 8 rows x (H_post | H_res) floats
  static constexpr int kSlot = kXSlot + kHSlot;
  static constexpr int kWarpScratch = sizeof(TX) == 2 ? 1 : 0;  // has the warp path
  static constexpr int kRowEpilogue = 0, kHalfRow = 0;
  static constexpr int warp_bytes(int depth) { return kYBytes + depth * kSlot; }
  // one pass (chunk step / 4, rows 8 (step % 4) ..) into ring slot `slot`
  __device__ __forceinline__ void prefetch(int64_t m0, int64_t n0, int step, int slot, int lane,
                                           unsigned char* ring, int64_t M) const {
    const int ch = step >> 2, p = step & 3;
    unsigned char* sl = ring + slot * kSlot;
    const int rq = lane >> 2, cq = lane & 3;
    const int64_t m = m0 + p * 8 + rq;
    const bool in = m < M;
    const int64_t mm = in ? m : 0;
    const TX* src = x + (size_t)mm * 4 * C + n0 + ch * 32 + cq * 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) cp_async16(sl + (rq * 4 + j) * 64 + cq * 16, src + (size_t)j * C, in ? 16 : 0);
    const float* hm = hmix + mm * kMapRows + 4;
    cp_async16(sl + kXSlot + rq * 80 + cq * 16, hm + 4 * cq, in ? 16 : 0);
    if (cq == 0) cp_async16(sl + kXSlot + rq * 80 + 64, hm + 16, in ? 16 : 0);
  }
  // all 32 lanes: rows m0 .. m0 + 31 (TMEM lane quarter of the warp), columns
  // n0 .. n0 + 127 of the accumulator at tensor-memory address `tacc`; DEPTH
  // ring slots, DEPTH - 1 passes in flight ahead of the one being mixed
  template <int DEPTH>
  __device__ __forceinline__ void warp_block(int64_t m0, int64_t n0, uint32_t tacc, int lane, unsigned char* scr,
                                             int64_t M) const {
    float* ys = reinterpret_cast<float*>(scr);
    unsigned char* ring = scr + kYBytes;
    const int rq = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int k = 0; k < DEPTH - 1; ++k) {
      prefetch(m0, n0, k, k, lane, ring, M);
      cp_async_commit();
    }
    float sc[8];
#pragma unroll 1
    for (int step = 0; step < 16; ++step) {
      const int ch = step >> 2, p = step & 3;
      if (p == 0) {
        float v[32];
        tc05::tmem_ld32(tacc + (uint32_t)(ch * 32), v);
        __syncwarp();  // previous chunk's staged rows fully read
        float* mine = ys + lane * kPitch;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(mine + 4 * k) = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + n0 + ch * 32 + cq * 8));
        const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + n0 + ch * 32 + cq * 8 + 4));
        sc[0] = s0.x; sc[1] = s0.y; sc[2] = s0.z; sc[3] = s0.w;
        sc[4] = s1.x; sc[5] = s1.y; sc[6] = s1.z; sc[7] = s1.w;
      }
      cp_async_wait<DEPTH - 2>();
      __syncwarp();
      const int r = p * 8 + rq;
      const int64_t m = m0 + r;
      const unsigned char* sl = ring + (step % DEPTH) * kSlot;
      if (m < M) {
        float h[20];
#pragma unroll
        for (int k = 0; k < 5; ++k) {
          const float4 t = *reinterpret_cast<const float4*>(sl + kXSlot + rq * 80 + 16 * k);
          h[4 * k] = t.x; h[4 * k + 1] = t.y; h[4 * k + 2] = t.z; h[4 * k + 3] = t.w;
        }
        const float4 y0 = *reinterpret_cast<const float4*>(ys + r * kPitch + cq * 8);
        const float4 y1 = *reinterpret_cast<const float4*>(ys + r * kPitch + cq * 8 + 4);
        const float f[8] = {y0.x * sc[0], y0.y * sc[1], y0.z * sc[2], y0.w * sc[3],
                            y1.x * sc[4], y1.y * sc[5], y1.z * sc[6], y1.w * sc[7]};
        float xf[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          unpack8(*reinterpret_cast<const uint4*>(sl + (rq * 4 + j) * 64 + cq * 16), xf[j], (const TX*)nullptr);
        const size_t base = (size_t)m * 4 * C + n0 + ch * 32 + cq * 8;
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const float* hr = h + 4 + 4 * o;
          const uint64_t h0 = f2_dup(hr[0]), h1 = f2_dup(hr[1]), h2 = f2_dup(hr[2]), h3 = f2_dup(hr[3]),
                         hp = f2_dup(h[o]);
          float out[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            // (((H0 x0 + H1 x1) + H2 x2) + H3 x3) + H_post f, two columns per instruction
            uint64_t a = f2_mul(h0, f2_pack(xf[0][e], xf[0][e + 1]));
            a = f2_fma(h1, f2_pack(xf[1][e], xf[1][e + 1]), a);
            a = f2_fma(h2, f2_pack(xf[2][e], xf[2][e + 1]), a);
            a = f2_fma(h3, f2_pack(xf[3][e], xf[3][e + 1]), a);
            a = f2_fma(hp, f2_pack(f[e], f[e + 1]), a);
            out[e] = __uint_as_float((uint32_t)a);
            out[e + 1] = __uint_as_float((uint32_t)(a >> 32));
          }
          store8(xo + base + (size_t)o * C, out);
        }
      }
      __syncwarp();  // the slot of step - 1 is free: refill it with step + DEPTH - 1
      if (step + DEPTH - 1 < 16) prefetch(m0, n0, step + DEPTH - 1, (step + DEPTH - 1) % DEPTH, lane, ring, M);
      cp_async_commit();
    }
    cp_async_wait<0>();
  }
};

// Router of the Hadamard MoE (src/model/moe.py:383-447) as the epilogue of
// h = u W1^T (N = 128 hidden units, one accumulator row per token):
// silu(h) rounded to the activation type (the operand type of the second
// layer), logits = silu(h) W2^T with W2 staged in shared memory as float
// ([hidden][expert], one broadcast 16-byte load per 4 experts), softmax,
// top-k (ties to the lower expert index) and the routing weights
// renormalised over the selected experts in ascending order.  Both epilogue
// warps of a tensor-memory lane quarter work on a row: the second takes
// hidden units 64..127 and hands its 16 partial logits to the first through
// shared memory (double-buffered by tile parity, one named barrier per
// quarter and tile), which adds them to its own over 0..63 and finishes.
template <typename TU>
struct EpiRouter {
  static constexpr int kWarpScratch = 0, kRowEpilogue = 1, kHalfRow = 0;
  static constexpr int E = 16, HID = 128;
  static constexpr int kRowScratch = E * HID * 4 + 2 * 128 * E * 4;  // W2 + partial-logit exchange
  const TU* w2;  // [E][HID]
  RouteRule rr;  // expert-selection rule
  uint8_t* mask;
  float* probs;
  float* weights;
  __host__ bool vec_ok() const { return true; }
  // all 256 epilogue threads (t = 0..255), before the first tile
  __device__ __forceinline__ void stage(float* ws, int t) const {
    for (int i = t; i < E * HID; i += 256) {
      const int e = i / HID, j = i - e * HID;
      ws[j * E + e] = to_f(w2[i]);
    }
  }
  // tacc: column 0 of this row's accumulator; half: which 64 hidden units;
  // r: the row within the tile (lane quarter x 32 + lane); par: tile parity
  __device__ __forceinline__ void row(int64_t m, uint32_t tacc, int half, int r, int par, float* ws,
                                      int64_t M) const {
    float l[E];
#pragma unroll
    for (int e = 0; e < E; ++e) l[e] = 0.f;
#pragma unroll 1
    for (int c = half * (HID / 2); c < (half + 1) * (HID / 2); c += 32) {
      float v[32];
      tc05::tmem_ld32(tacc + (uint32_t)c, v);
#pragma unroll 4
      for (int j = 0; j < 32; ++j) {
        const float h = to_f(from_f<TU>(siluf_(v[j])));
        const float4* wr = reinterpret_cast<const float4*>(ws + (c + j) * E);
#pragma unroll
        for (int q = 0; q < E / 4; ++q) {
          const float4 w = wr[q];
          l[4 * q] = fmaf(h, w.x, l[4 * q]);
          l[4 * q + 1] = fmaf(h, w.y, l[4 * q + 1]);
          l[4 * q + 2] = fmaf(h, w.z, l[4 * q + 2]);
          l[4 * q + 3] = fmaf(h, w.w, l[4 * q + 3]);
        }
      }
    }
    float4* xg = reinterpret_cast<float4*>(ws + E * HID + (par * 128 + r) * E);
    if (half) {
#pragma unroll
      for (int q = 0; q < E / 4; ++q) xg[q] = make_float4(l[4 * q], l[4 * q + 1], l[4 * q + 2], l[4 * q + 3]);
    }
    asm volatile("bar.sync %0, 64;\n" ::"r"(2 + (r >> 5)) : "memory");  // the quarter's two warps
    if (half) return;
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      const float4 o = xg[q];
      l[4 * q] += o.x;
      l[4 * q + 1] += o.y;
      l[4 * q + 2] += o.z;
      l[4 * q + 3] += o.w;
    }
    if (m >= M) return;
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, l[e]);
    float p[E], sum = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      p[e] = expf(l[e] - mx);
      sum += p[e];
    }
#pragma unroll
    for (int e = 0; e < E; ++e) p[e] = __fdiv_rn(p[e], sum);
    uint32_t chosen = 0;
    for (int k = 0; k < rr.kmax; ++k) {
      int best = -1;
      float bv = -1.f;
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (!((chosen >> e) & 1u) && p[e] > bv) {
          bv = p[e];
          best = e;
        }
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
    float wv[E];
    uint32_t mk[E / 4];
#pragma unroll
    for (int q = 0; q < E / 4; ++q) mk[q] = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const bool on = (chosen >> e) & 1u;
      wv[e] = on ? __fdiv_rn(p[e], wsum) : 0.f;
      mk[e >> 2] |= (on ? 1u : 0u) << (8 * (e & 3));
    }
    float4* wo = reinterpret_cast<float4*>(weights + m * E);
    float4* po = reinterpret_cast<float4*>(probs + m * E);
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      wo[q] = make_float4(wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]);
      po[q] = make_float4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
    }
    *reinterpret_cast<uint4*>(mask + m * E) = make_uint4(mk[0], mk[1], mk[2], mk[3]);
  }
};

}  // namespace octo

template <typename TA, class Epi>
__global__ void __launch_bounds__(octo::NT)
octo_gemm_kernel(const TA* __restrict__ a, int64_t M, int K, const octo::TE<TA>* __restrict__ whi,
                 const octo::TE<TA>* __restrict__ wlo, int64_t N, Epi epi) {
  using namespace octo;
  using W = TE<TA>;
  constexpr bool SPLIT = std::is_same<TA, float>::value;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int wm = warp & 1, wn = warp >> 1;  // 2 x 4 warps: 64 rows x 32 columns each
  const int nk = (K + BK - 1) / BK;
  const bool lo = wlo != nullptr;
  auto As = [&](int st) { return reinterpret_cast<TA*>(smem_raw + st * stage_bytes<TA>()); };
  auto Wh = [&](int st) {
    return reinterpret_cast<W*>(smem_raw + st * stage_bytes<TA>() + BM * LD * (int)sizeof(TA));
  };
  auto Wl = [&](int st) { return Wh(st) + BN * LD; };
  auto load_stage = [&](int kt, int st) {
    const int k0 = kt * BK;
    constexpr int AV = 16 / (int)sizeof(TA);  // A elements per 16-byte chunk
    TA* as = As(st);
    for (int i = tid; i < BM * (BK / AV); i += NT) {
      const int r = i / (BK / AV), c = (i % (BK / AV)) * AV;
      const int64_t m = m0 + r;
      const bool in = m < M && k0 + c < K;  // K is a multiple of 8: chunks are all in or all out
      cp_async16(as + r * LD + c, a + (in ? (size_t)m * K + k0 + c : 0), in ? 16 : 0);
    }
    W* wh = Wh(st);
    W* wl = Wl(st);
    for (int i = tid; i < BN * (BK / 8); i += NT) {
      const int r = i / (BK / 8), c = (i % (BK / 8)) * 8;
      const int64_t n = n0 + r;
      const bool in = n < N && k0 + c < K;
      const size_t off = in ? (size_t)n * K + k0 + c : 0;
      cp_async16(wh + r * LD + c, whi + off, in ? 16 : 0);
      if (lo) cp_async16(wl + r * LD + c, wlo + off, in ? 16 : 0);
    }
  };
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (st < nk) load_stage(st, st);
    cp_async_commit();
  }
  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;

  for (int kt = 0; kt < nk; ++kt) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (kt + STAGES - 1 < nk) load_stage(kt + STAGES - 1, (kt + STAGES - 1) % STAGES);
    cp_async_commit();
    const int st = kt % STAGES;
    const TA* as = As(st);
    const W* wh = Wh(st);
    const W* wl = Wl(st);
#pragma unroll
    for (int kk = 0; kk < BK; kk += 16) {
      uint32_t ah[4][4], al[4][4];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int r = wm * 64 + mi * 16;
        if constexpr (SPLIT) {
          const float* af = reinterpret_cast<const float*>(as);
          const float2 v0 = *reinterpret_cast<const float2*>(af + (r + g) * LD + kk + 2 * t4);
          const float2 v1 = *reinterpret_cast<const float2*>(af + (r + g + 8) * LD + kk + 2 * t4);
          const float2 v2 = *reinterpret_cast<const float2*>(af + (r + g) * LD + kk + 8 + 2 * t4);
          const float2 v3 = *reinterpret_cast<const float2*>(af + (r + g + 8) * LD + kk + 8 + 2 * t4);
          split_bf16(v0.x, v0.y, ah[mi][0], al[mi][0]);
          split_bf16(v1.x, v1.y, ah[mi][1], al[mi][1]);
          split_bf16(v2.x, v2.y, ah[mi][2], al[mi][2]);
          split_bf16(v3.x, v3.y, ah[mi][3], al[mi][3]);
        } else {
          ldsm_x4(ah[mi], as + (r + (lane & 15)) * LD + kk + (lane >> 4) * 8);
        }
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int rn = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int cn = kk + ((lane >> 3) & 1) * 8;
        uint32_t bh[4], bl[4];
        ldsm_x4(bh, wh + rn * LD + cn);
        if (lo) ldsm_x4(bl, wl + rn * LD + cn);
#pragma unroll
        for (int mi = 0; mi < 4; ++mi) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float* c = acc[mi][2 * np + h];
            if constexpr (SPLIT) mma16<W>(c, al[mi], bh[2 * h], bh[2 * h + 1]);
            if (lo) mma16<W>(c, ah[mi], bl[2 * h], bl[2 * h + 1]);
            mma16<W>(c, ah[mi], bh[2 * h], bh[2 * h + 1]);
          }
        }
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      const int64_t n = n0 + wn * 32 + ni * 8 + 2 * t4;
      if (n >= N) continue;  // N is even: the pair (n, n + 1) is all in or all out
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int64_t m = m0 + wm * 64 + mi * 16 + g + hr * 8;
        if (m < M) epi(m, n, acc[mi][ni][2 * hr], acc[mi][ni][2 * hr + 1]);
      }
    }
}

// ---------------------------------------------------------------------------
// The same GEMMs on the 5th-generation tensor cores (16-bit x, no W_lo).
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0     TMA producer: A [128 x 64] and B [256 x 64] tiles (128-byte
//              swizzle) into a 4-stage shared-memory ring (48 KB a stage);
//   warp 1     allocates all 512 TMEM columns and issues tcgen05.mma
//              (M128 N256 K16, fp32 accumulators), freeing each ring stage
//              with tcgen05.commit; two 256-column accumulators alternate
//              between tiles;
//   warps 2-9  epilogue, two warps per TMEM lane quarter (one per half of
//              the 256 columns): tcgen05.ld of their 32 accumulator rows, 32
//              columns at a time, into the fused epilogue, then release the
//              accumulator so the MMAs of the tile after next can start.
// So the epilogue of one tile overlaps the MMAs of the next.  Tiles are
// walked N-fastest so CTAs running at the same time share A rows in L2.
// ---------------------------------------------------------------------------
namespace octo_tc {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, ACC_COLS = 256, TMEM_COLS = 512;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NTHREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /* alignment slack */ + 256 /* barriers */;
}  // namespace octo_tc

// Epilogues with a TMA-store path declare kTmaStore = 1 (scale32, out_t).
template <class E, class = void>
struct TmaStoreOf {
  static constexpr int value = 0;
};
template <class E>
struct TmaStoreOf<E, std::void_t<decltype(E::kTmaStore)>> {
  static constexpr int value = E::kTmaStore;
};

// Launch shape: mainloop stages, epilogue ring depth and shared memory.  An
// epilogue with a warp path trades mainloop stages for in-flight stream
// rows: 2 stages and a 4-slot ring for K <= 512 (short mainloops), else 3 and 2.
template <class Epi>
struct OctoTcShape {
  int stages, depth, smem;
  explicit OctoTcShape(int K) {
    if constexpr (Epi::kWarpScratch > 0) {
      stages = K <= 512 ? 2 : 3;
      depth = K <= 512 ? 4 : 2;
      smem = scratch_off(stages) + 8 * Epi::warp_bytes(depth) + 1024;
    } else if constexpr (Epi::kRowEpilogue > 0) {
      stages = 3;
      depth = 0;
      smem = scratch_off(stages) + Epi::kRowScratch + 1024;
    } else if constexpr (Epi::kHalfRow > 0) {
      stages = octo_tc::STAGES;
      depth = 0;
      smem = scratch_off(stages) + Epi::kRowScratch + 1024;
    } else if constexpr (TmaStoreOf<Epi>::value > 0) {
      // per epilogue warp two 32 x 32 16-bit staging blocks (64-byte
      // swizzle), 1024-byte aligned after the barriers
      stages = octo_tc::STAGES;
      depth = 0;
      smem = tma_stage_off(stages) + 8 * 2 * 2048 + 1024;
    } else {
      stages = octo_tc::STAGES;
      depth = 0;
      smem = scratch_off(stages) + 1024;
    }
  }
  __host__ __device__ static int tma_stage_off(int stages) { return (scratch_off(stages) + 1023) & ~1023; }
  __host__ __device__ static int scratch_off(int stages) { return stages * octo_tc::STAGE_BYTES + 256; }
};

// Set when a bounded wait of a tcgen05 kernel in this file gave up.
__device__ int g_tc05_error;

template <typename TA, class Epi, int BNT>
__global__ void __launch_bounds__(octo_tc::NTHREADS, 1)
octo_gemm_tc05_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_y, int64_t M, int K, int64_t N, Epi epi, int vec,
                      int nstage, int depth) {
  using namespace octo_tc;
  using namespace tc05;
  // BNT: the CTA tile's width (256; 64 for few-row GEMMs, so that more CTAs
  // share the columns); the stage keeps the 256-wide layout's offsets
  constexpr int BN = BNT, B_BYTES = BN * BK * 2;
  static_assert(BN == 256 || (BN == 64 && Epi::kRowEpilogue == 0 && Epi::kWarpScratch == 0), "tile width");
  const int STAGES = nstage;  // mainloop stages of this launch (2..4)
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (K + BK - 1) / BK;
  const int64_t mt = (M + BM - 1) / BM, ntl = (N + BN - 1) / BN, tiles = mt * ntl;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t IDESC = idesc_f16(std::is_same<TA, __nv_bfloat16>::value, BM, BN);

  if (warp == 0) {
    if (lane == 0) {
      int64_t g = 0;  // k-iterations issued by this CTA
      for (int64_t t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (int)((t / ntl) * BM), n0 = (int)((t % ntl) * BN);
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int st = (int)(g % STAGES);
          if (g >= STAGES && !mbar_wait(&empty[st], (uint32_t)(((g / STAGES) - 1) & 1))) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[st], A_BYTES + B_BYTES);
          tma_load_2d(smem + st * STAGE_BYTES, &tma_a, &full[st], kt * BK, m0);
          tma_load_2d(smem + st * STAGE_BYTES + A_BYTES, &tma_b, &full[st], kt * BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int64_t g = 0;
      int i = 0;  // tiles of this CTA
      for (int64_t t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&acc_empty[b], (uint32_t)(((i >> 1) - 1) & 1))) {
          *abort_flag = 1;
          break;
        }
        fence_after_sync();
        const uint32_t d = tmem + (uint32_t)(b * ACC_COLS);
        bool ok = true;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int st = (int)(g % STAGES);
          if (!mbar_wait(&full[st], (uint32_t)((g / STAGES) & 1))) {
            ok = false;
            break;
          }
          fence_after_sync();
          const uint32_t a0 = smem_u32(smem + st * STAGE_BYTES);
          const uint64_t ad = sw128_desc(a0), bd = sw128_desc(a0 + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_f16(d, ad + 2 * k, bd + 2 * k, IDESC, (kt | k) != 0);
          umma_commit(&empty[st]);
        }
        umma_commit(&acc_full[b]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
  } else {
    // epilogue warps 2..9: TMEM lane quarter (warp % 4) holds accumulator rows
    // 32 (warp % 4) ..; warps 2-5 take columns 0..127, warps 6-9 128..255
    const int q = warp & 3, half = (warp - 2) >> 2;
    float* rowscr = nullptr;
    if constexpr (Epi::kRowEpilogue > 0 || Epi::kHalfRow > 0) {
      rowscr = reinterpret_cast<float*>(smem + OctoTcShape<Epi>::scratch_off(STAGES));
      if (Epi::kRowEpilogue > 0 || vec == 2) epi.stage(rowscr, threadIdx.x - 64);
      asm volatile("bar.sync 1, 256;\n" ::: "memory");  // the 8 epilogue warps
    }
    // TMA-store form (vec == 3): each warp's two 32 x 32 staging blocks
    unsigned char* stg = smem + OctoTcShape<Epi>::tma_stage_off(STAGES) + (warp - 2) * 4096;
    int nst = 0;  // blocks this warp has stored
    int i = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      if (!mbar_wait(&acc_full[b], (uint32_t)((i >> 1) & 1)) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      fence_after_sync();
      const int64_t m = (t / ntl) * BM + q * 32 + lane, n0 = (t % ntl) * BN + half * (BN / 2);
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * ACC_COLS + half * (BN / 2));
      bool done = false;
      if constexpr (TmaStoreOf<Epi>::value > 0) {
        if (vec == 3) {
          // lane = row: scaled, rounded 32-column block into a staging block
          // (16-byte chunk j of row r at chunk j ^ ((r >> 1) & 3), the 64-byte
          // swizzle of the output map), then one lane stores the block; a
          // block is rewritten only after the store issued two blocks
          // earlier has read it.  The map clips rows >= M and columns >= N.
          using TO = typename Epi::out_t;
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 32, ++nst) {
            float v[32];
            tmem_ld32(base + (uint32_t)c, v);
            const int64_t n = n0 + c;
            if (n < N) epi.scale32(n, v);
            unsigned char* blk = stg + (nst & 1) * 2048;
            if (lane == 0) bulk_wait_read1();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 w;
              w.x = pack2<TO>(v[8 * j], v[8 * j + 1]);
              w.y = pack2<TO>(v[8 * j + 2], v[8 * j + 3]);
              w.z = pack2<TO>(v[8 * j + 4], v[8 * j + 5]);
              w.w = pack2<TO>(v[8 * j + 6], v[8 * j + 7]);
              *reinterpret_cast<uint4*>(blk + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = w;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0 && n < N && m < M) {  // m: the warp's first row (lane 0)
              tma_store_2d(&tma_y, blk, (int)n, (int)m);
              bulk_commit();
            }
          }
          done = true;
        }
      }
      if constexpr (Epi::kRowEpilogue > 0) {  // N <= BN / 2: both halves split the first 128 columns
        epi.row(m, base - (uint32_t)(half * (BN / 2)), half, q * 32 + lane, i & 1, rowscr, M);
        done = true;
      }
      if constexpr (Epi::kHalfRow > 0 && BN == 256) {
        if (vec == 2 && n0 + BN / 2 <= N) {  // uniform over the warp
          epi.half_row(m, n0, base, rowscr, M);
          done = true;
        }
      }
      if constexpr (Epi::kWarpScratch > 0) {
        if (vec && n0 + BN / 2 <= N) {  // uniform over the warp
          unsigned char* scr =
              smem + OctoTcShape<Epi>::scratch_off(STAGES) + (warp - 2) * Epi::warp_bytes(depth);
          if (depth == 4)
            epi.template warp_block<4>(m - lane, n0, base, lane, scr, M);
          else
            epi.template warp_block<2>(m - lane, n0, base, lane, scr, M);
          done = true;
        }
      }
      if constexpr (Epi::kRowEpilogue == 0) {
#pragma unroll 1
        for (int c = 0; c < BN / 2 && !done; c += 32) {
          float v[32];
          tmem_ld32(base + (uint32_t)c, v);
          const int64_t n = n0 + c;
          if (m < M && n < N) {
            if (vec && n + 32 <= N) {
              epi.chunk32(m, n, v);
            } else {
#pragma unroll
              for (int j = 0; j < 32; j += 2)
                if (n + j < N) epi(m, n + j, v[j], v[j + 1]);
            }
          }
        }
      }
      (void)done;
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (lane == 0 && nst > 0) bulk_wait_all();  // the stores are done before the CTA exits
  }
  __syncwarp();
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_tc05_error, (int)WALSH_ERR_TIMEOUT);
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// 1 when the tcgen05 path ran, 0 when it does not apply (caller falls back),
// negative on a launch error.
// Plain-epilogue GEMMs store their output through shared memory by TMA
// when on (walsh_octo_set_tma_store).
int g_octo_tma_store = 1;

template <typename TA, class Epi, int BNT>
static int launch_octo_tc05_bn(const void* a, int64_t M, int K, const void* w, int64_t N, const Epi& epi,
                               cudaStream_t s) {
  using namespace octo_tc;
  if (M < 1 || M > 2147483647LL || N > 2147483647LL) return 0;
  constexpr bool BF = std::is_same<TA, __nv_bfloat16>::value;
  CUtensorMap ma, mb, my;
  if (!make_tile_map(&ma, a, BF, M, K, octo_tc::BK, BM) || !make_tile_map(&mb, w, BF, N, K, octo_tc::BK, BNT)) return 0;
  memset(&my, 0, sizeof(my));
  auto kern = octo_gemm_tc05_kernel<TA, Epi, BNT>;
  const OctoTcShape<Epi> shp(K);
  const int SMEM_B = shp.smem;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_B) != cudaSuccess)
    return launch_status();
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                   cudaSuccess)
      sms = 148;
  }
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BNT - 1) / BNT);
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  int vec = epi.vec_ok() ? 1 : 0;  // 2: the epilogue's row path (half_row) applies
  if constexpr (Epi::kHalfRow > 0 && BNT == 256) {
    if (epi.half_row_ok()) vec = 2;
  }
  if constexpr (TmaStoreOf<Epi>::value > 0) {
    // 3: scaled blocks leave through shared memory by TMA stores
    if (g_octo_tma_store && epi.tma_ok() && std::is_same<typename Epi::out_t, TA>::value &&
        make_store_map(&my, epi.y, BF, M, N))
      vec = 3;
  }
  kern<<<grid, NTHREADS, SMEM_B, s>>>(ma, mb, my, M, K, N, epi, vec, shp.stages, shp.depth);
  const int st = launch_status();
  return st == WALSH_OK ? 1 : st;
}

// Few-row GEMMs (batched decode: M of a few hundred) whose 256-wide tiles
// would occupy a small fraction of the SMs run with 64-wide tiles; epilogues
// with a row or warp-cooperative path keep the 256-wide tile.
int g_octo_narrow = 1;
template <typename TA, class Epi>
static int launch_octo_tc05(const void* a, int64_t M, int K, const void* w, int64_t N, const Epi& epi,
                            cudaStream_t s) {
  using namespace octo_tc;
  if constexpr (Epi::kRowEpilogue == 0 && Epi::kWarpScratch == 0) {
    const int64_t wide = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    if (g_octo_narrow && wide * 4 <= 148 && N >= 128)
      return launch_octo_tc05_bn<TA, Epi, 64>(a, M, K, w, N, epi, s);
  }
  return launch_octo_tc05_bn<TA, Epi, 256>(a, M, K, w, N, epi, s);
}

template <typename TA, class Epi>
static int launch_octo(const void* a, int64_t M, int K, const void* whi, const void* wlo, int64_t N, const Epi& epi,
                       cudaStream_t s) {
  using namespace octo;
  if constexpr (!std::is_same<TA, float>::value) {
    if (!wlo && octo_tc05_enabled()) {
      const int r = launch_octo_tc05<TA>(a, M, K, whi, N, epi, s);
      if (r != 0) return r > 0 ? WALSH_OK : r;
    }
  }
  auto kern = octo_gemm_kernel<TA, Epi>;
  const int smem = smem_bytes<TA>();
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status();
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  kern<<<grid, NT, smem, s>>>((const TA*)a, M, K, (const TE<TA>*)whi, (const TE<TA>*)wlo, N, epi);
  return launch_status();
}

// y [M, N] float = a [M, K] w^T (bf16 a and w), on the tcgen05 kernel when it
// applies, else the mma.sync kernel.  Internal: the channel-modulation MLP's
// first layer (its fp32 input split into bf16 hi, mid and lo rows).
int gemm_bf16_f32out(const __nv_bfloat16* a, int64_t M, int K, const __nv_bfloat16* w, int64_t N, float* y,
                     cudaStream_t s) {
  return launch_octo<__nv_bfloat16>(a, M, K, w, nullptr, N, octo::EpiStoreF32{y, N}, s);
}

// Shared argument checks: x dtype selects the weight dtype (fp16 W for fp16
// x, bf16 W otherwise); a W_lo correction matrix is only used with fp32 x.
static walsh_status octo_check(const void* x, int dtype, int64_t M, int K, const void* whi, const void* wlo,
                               int w_dtype, int64_t N) {
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(x && whi);
  WALSH_CHECK_SHAPE(M >= 0 && K > 0 && N > 0 && K % 8 == 0 && N % 2 == 0);
  WALSH_CHECK_SHAPE((M + octo::BM - 1) / octo::BM <= 2147483647LL && (N + octo::BN - 1) / octo::BN <= 65535);
  const int want = dtype == WALSH_F16 ? WALSH_F16 : WALSH_BF16;
  if (w_dtype != want) return WALSH_ERR_DTYPE;
  if (wlo && dtype != WALSH_F32) return WALSH_ERR_ARG;
  if ((((uintptr_t)x) | ((uintptr_t)whi) | ((uintptr_t)wlo)) & 15u) return WALSH_ERR_ALIGN;
  return WALSH_OK;
}

#define WALSH_OCTO_DISPATCH(dtype, TA, ...)                         \
  ((dtype) == WALSH_F32    ? ([&] { using TA = float; return __VA_ARGS__; }())   \
   : (dtype) == WALSH_BF16 ? ([&] { using TA = __nv_bfloat16; return __VA_ARGS__; }()) \
                           : ([&] { using TA = __half; return __VA_ARGS__; }()))

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_octo_linear_fwd(const void* x, int dtype, int64_t M, int K, const void* w_hi,
                                              const void* w_lo, int w_dtype, int64_t N, const float* scale, void* y,
                                              void* stream) {
  if (int e = injected("octo_linear_fwd")) return e;
  if (walsh_status st = octo_check(x, dtype, M, K, w_hi, w_lo, w_dtype, N)) return st;
  WALSH_CHECK_ARG(scale && y);
  if (((uintptr_t)y) & 7u) return WALSH_ERR_ALIGN;
  if (M == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  return WALSH_OCTO_DISPATCH(dtype, TA,
                             launch_octo<TA>(x, M, K, w_hi, w_lo, N, octo::EpiPlain<TA>{scale, (TA*)y, N}, s));
}

extern "C" walsh_status walsh_hadamard_linear_dense_fwd(const void* x, int dtype, int64_t ntok, int features,
                                                        const void* w_dense, const float* scale, void* y,
                                                        void* stream) {
  if (int e = injected("hadamard_linear_dense_fwd")) return e;
  WALSH_CHECK_SHAPE(features == 512 || features == 2048);
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  if (walsh_status st = octo_check(x, dtype, ntok, features, w_dense, nullptr, dtype, features)) return st;
  WALSH_CHECK_ARG(scale && y);
  if ((((uintptr_t)y) | ((uintptr_t)scale)) & 15u) return WALSH_ERR_ALIGN;
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == WALSH_BF16)
    return launch_octo<__nv_bfloat16>(x, ntok, features, w_dense, nullptr, features,
                                      octo::EpiPlain<__nv_bfloat16>{scale, (__nv_bfloat16*)y, features}, s);
  return launch_octo<__half>(x, ntok, features, w_dense, nullptr, features,
                             octo::EpiPlain<__half>{scale, (__half*)y, features}, s);
}

extern "C" walsh_status walsh_moe_router_tc_fwd(const void* u, int dtype, int64_t ntok, const void* w1,
                                               const void* w2, int top_k, uint8_t* mask, float* probs,
                                               float* weights, const walsh_moe_routing* routing, void* stream) {
  if (int e = injected("moe_router_tc_fwd")) return e;
  WALSH_CHECK_ARG(u && w1 && w2 && mask && probs && weights);
  WALSH_CHECK_SHAPE(ntok >= 0 && ntok <= 2147483647LL && top_k >= 1 && top_k <= 16);
  RouteRule rr;
  if (int e = make_route_rule(top_k, routing, &rr)) return e;
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  if ((((uintptr_t)u) | ((uintptr_t)w1) | ((uintptr_t)mask) | ((uintptr_t)probs) | ((uintptr_t)weights)) & 15u)
    return WALSH_ERR_ALIGN;
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  int r;
  if (dtype == WALSH_BF16)
    r = launch_octo_tc05<__nv_bfloat16>(u, ntok, 512, w1, 128,
                                        octo::EpiRouter<__nv_bfloat16>{(const __nv_bfloat16*)w2, rr, mask, probs,
                                                                       weights},
                                        s);
  else
    r = launch_octo_tc05<__half>(u, ntok, 512, w1, 128,
                                 octo::EpiRouter<__half>{(const __half*)w2, rr, mask, probs, weights}, s);
  return r == 1 ? WALSH_OK : (r == 0 ? WALSH_ERR_SHAPE : r);
}

extern "C" walsh_status walsh_octo_qkv_fwd(const void* u, int dtype, int B, int T, int C, int n_head,
                                           const void* w_hi, const void* w_lo, int w_dtype, const float* scale,
                                           const float* rope_cos, const float* rope_sin, int n_pos, int start_pos,
                                           void* q, void* k_cache, void* v_cache, int ctx, void* stream) {
  if (int e = injected("octo_qkv_fwd")) return e;
  WALSH_CHECK_SHAPE(B > 0 && T > 0 && C > 0 && n_head > 0 && C % n_head == 0);
  const int hd = C / n_head;
  WALSH_CHECK_SHAPE(hd % 2 == 0 && start_pos >= 0 && start_pos + T <= ctx && T <= n_pos);
  const int64_t M = (int64_t)B * T;
  WALSH_CHECK_SHAPE(M <= 2147483647LL);  // the epilogue's index math is 32-bit
  if (walsh_status st = octo_check(u, dtype, M, C, w_hi, w_lo, w_dtype, 3 * (int64_t)C)) return st;
  WALSH_CHECK_ARG(scale && rope_cos && rope_sin && q && k_cache && v_cache);
  if ((((uintptr_t)q) | ((uintptr_t)k_cache) | ((uintptr_t)v_cache)) & 7u) return WALSH_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  auto log2_or_neg = [](int v) {
    int k = 0;
    while ((1 << k) < v) ++k;
    return (1 << k) == v ? k : -1;
  };
  const int c_shift = log2_or_neg(C), hd_shift = log2_or_neg(hd);
  return WALSH_OCTO_DISPATCH(dtype, TA,
                             launch_octo<TA>(u, M, C, w_hi, w_lo, 3 * (int64_t)C,
                                             octo::EpiQkv<TA>{scale, (TA*)q, (TA*)k_cache, (TA*)v_cache, rope_cos,
                                                              rope_sin, T, n_head, hd, C, ctx, start_pos, c_shift,
                                                              hd_shift},
                                             s));
}

extern "C" walsh_status walsh_octo_swiglu_fwd(const void* u, int dtype, int64_t M, int K, const void* w_hi,
                                              const void* w_lo, int w_dtype, const float* scale, int64_t hidden,
                                              void* h, void* stream) {
  if (int e = injected("octo_swiglu_fwd")) return e;
  WALSH_CHECK_SHAPE(hidden > 0);
  if (walsh_status st = octo_check(u, dtype, M, K, w_hi, w_lo, w_dtype, 2 * hidden)) return st;
  WALSH_CHECK_ARG(scale && h);
  if (M == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  return WALSH_OCTO_DISPATCH(dtype, TA,
                             launch_octo<TA>(u, M, K, w_hi, w_lo, 2 * hidden,
                                             octo::EpiSwiglu<TA>{scale, (TA*)h, hidden}, s));
}

extern "C" walsh_status walsh_octo_post_fwd(const void* a, int dtype, int64_t M, int K, const void* w_hi,
                                            const void* w_lo, int w_dtype, const float* scale, int C, const void* x,
                                            int x_dtype, const float* hmix, void* x_out, void* stream) {
  if (int e = injected("octo_post_fwd")) return e;
  WALSH_CHECK_SHAPE(C > 0);
  if (walsh_status st = octo_check(a, dtype, M, K, w_hi, w_lo, w_dtype, C)) return st;
  WALSH_CHECK_ARG(scale && x && hmix && x_out);
  WALSH_CHECK_DTYPE(x_dtype);
  if ((((uintptr_t)x) | ((uintptr_t)x_out)) & 7u) return WALSH_ERR_ALIGN;
  if (M == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (x_dtype == WALSH_F16)
    return WALSH_OCTO_DISPATCH(dtype, TA,
                               launch_octo<TA>(a, M, K, w_hi, w_lo, C,
                                               octo::EpiPost<__half>{scale, (const __half*)x, hmix, (__half*)x_out, C},
                                               s));
  if (x_dtype == WALSH_F32)
    return WALSH_OCTO_DISPATCH(dtype, TA,
                               launch_octo<TA>(a, M, K, w_hi, w_lo, C,
                                               octo::EpiPost<float>{scale, (const float*)x, hmix, (float*)x_out, C},
                                               s));
  return WALSH_OCTO_DISPATCH(
      dtype, TA,
      launch_octo<TA>(a, M, K, w_hi, w_lo, C,
                      octo::EpiPost<__nv_bfloat16>{scale, (const __nv_bfloat16*)x, hmix, (__nv_bfloat16*)x_out, C},
                      s));
}

// Exercises the bounded-wait path of the tcgen05 kernels: one thread waits on
// an mbarrier that nothing arrives at, gives up after `budget` clock cycles
// and records WALSH_ERR_TIMEOUT like a stalled pipeline would.
__global__ void tc05_wait_selftest_kernel(long long budget) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc05::mbar_init(&bar, 1);
    tc05::fence_barrier_init();
    if (!tc05::mbar_wait(&bar, 0, budget)) atomicExch(&g_tc05_error, (int)WALSH_ERR_TIMEOUT);
  }
}

extern "C" walsh_status walsh_tc05_wait_selftest(long long budget_cycles, void* stream) {
  WALSH_CHECK_ARG(budget_cycles > 0 && budget_cycles <= 4000000000LL);
  tc05_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(budget_cycles);
  return launch_status();
}

extern "C" int walsh_octo_set_mainloop(int tcgen05) {
  const int prev = g_octo_tc05;
  g_octo_tc05 = tcgen05 ? 1 : 0;
  return prev;
}

extern "C" int walsh_octo_set_narrow(int on) {
  const int prev = walsh::g_octo_narrow;
  if (on >= 0) walsh::g_octo_narrow = on ? 1 : 0;
  return prev;
}

extern "C" int walsh_octo_set_tma_store(int on) {
  const int prev = walsh::g_octo_tma_store;
  if (on >= 0) walsh::g_octo_tma_store = on ? 1 : 0;
  return prev;
}

namespace walsh {
int attn_tc05_error(int reset);  // attention_tc.cu
int moe_tc05_error(int reset);   // moe.cu
}

extern "C" int walsh_tc05_error(int reset) {
  const int va = walsh::attn_tc05_error(reset);
  const int vm = walsh::moe_tc05_error(reset);
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc05_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_tc05_error, &zero, sizeof(int));
  }
  return v ? v : (va ? va : vm);
}
