// Shared device/host helpers for libwalsh (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "walsh.h"

namespace walsh {

constexpr int kGroups = 32;      // Hadamard algebra dimension
constexpr int kStreams = 4;      // mHC residual streams supported by the fused kernels
constexpr int kMapRows = 24;     // phi rows: pre(4) | post(4) | res(16)
constexpr int kExpertHidden = 128;
constexpr int kBlock = 32;       // Hadamard block width (experts, channel modulation)

// ---- activation storage types -------------------------------------------------
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
// fp16 stores saturate at +-65504 rather than overflowing to inf
template <> __device__ __forceinline__ __half from_f<__half>(float v) {
  return __float2half_rn(fminf(fmaxf(v, -65504.f), 65504.f));
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// Expert-selection rule of the MoE router.  Experts are taken in descending
// probability (ties to the lower index), at most kmax of them; the k-th pick
// (k >= kmin, counted from 0) is not taken when its probability is not above
// thr.  The reference's top-k is kmin = kmax (never stops early); the
// threshold rule keeps every expert with p > thr, at least kmin, at most kmax.
struct RouteRule {
  int kmax, kmin;
  float thr;
  __host__ __device__ __forceinline__ bool stop(int k, float p) const { return k >= kmin && !(p > thr); }
};

// Host: the rule for a top_k argument and an optional walsh_moe_routing.
static inline int make_route_rule(int top_k, const walsh_moe_routing* r, RouteRule* rr) {
  rr->kmax = top_k;
  rr->kmin = top_k;
  rr->thr = -1.f;
  if (r == nullptr || r->mode == WALSH_ROUTE_TOPK) return WALSH_OK;
  if (r->mode != WALSH_ROUTE_THRESHOLD) return WALSH_ERR_ARG;
  if (r->min_experts < 1 || r->min_experts > top_k || !(r->threshold >= 0.f && r->threshold <= 1.f))
    return WALSH_ERR_ARG;
  rr->kmin = r->min_experts;
  rr->thr = r->threshold;
  return WALSH_OK;
}

// 8 consecutive elements <-> float[8] (16-byte accesses for 16-bit types, 2 x 16 for float).
__device__ __forceinline__ void load8(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename T16>
__device__ __forceinline__ void load8_16(const T16* p, float* v) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    T16 lo, hi;
    const uint16_t l = (uint16_t)(w[i] & 0xffffu), h = (uint16_t)(w[i] >> 16);
    memcpy(&lo, &l, 2);
    memcpy(&hi, &h, 2);
    v[2 * i] = to_f(lo);
    v[2 * i + 1] = to_f(hi);
  }
}
// 8 16-bit values already in registers (a 16-byte vector) to float; the
// pointer argument only selects the element type.
template <typename T16>
__device__ __forceinline__ void unpack8(const uint4 q, float* v, const T16*) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    T16 lo, hi;
    const uint16_t l = (uint16_t)(w[i] & 0xffffu), h = (uint16_t)(w[i] >> 16);
    memcpy(&lo, &l, 2);
    memcpy(&hi, &h, 2);
    v[2 * i] = to_f(lo);
    v[2 * i + 1] = to_f(hi);
  }
}
// 8 consecutive elements held raw in registers (loaded ahead of use), then
// converted to float: one 16-byte vector for 16-bit types, two for float.
template <typename T>
struct Vec8 {
  uint4 a;
};
template <>
struct Vec8<float> {
  float4 a, b;
};
template <typename T>
__device__ __forceinline__ Vec8<T> ld_vec8(const T* p) {
  Vec8<T> r;
  r.a = *reinterpret_cast<const uint4*>(p);
  return r;
}
template <>
__device__ __forceinline__ Vec8<float> ld_vec8<float>(const float* p) {
  Vec8<float> r;
  r.a = *reinterpret_cast<const float4*>(p);
  r.b = *reinterpret_cast<const float4*>(p + 4);
  return r;
}
template <typename T>
__device__ __forceinline__ void unpack_vec8(const Vec8<T>& r, float* v) {
  unpack8(r.a, v, (const T*)nullptr);
}
template <>
__device__ __forceinline__ void unpack_vec8<float>(const Vec8<float>& r, float* v) {
  v[0] = r.a.x; v[1] = r.a.y; v[2] = r.a.z; v[3] = r.a.w;
  v[4] = r.b.x; v[5] = r.b.y; v[6] = r.b.z; v[7] = r.b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) { load8_16(p, v); }
__device__ __forceinline__ void load8(const __half* p, float* v) { load8_16(p, v); }

__device__ __forceinline__ void store8(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
template <typename T16>
__device__ __forceinline__ void store8_16(T16* p, const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T16 lo = from_f<T16>(v[2 * i]), hi = from_f<T16>(v[2 * i + 1]);
    uint16_t l, h;
    memcpy(&l, &lo, 2);
    memcpy(&h, &hi, 2);
    w[i] = (uint32_t)l | ((uint32_t)h << 16);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) { store8_16(p, v); }
__device__ __forceinline__ void store8(__half* p, const float* v) { store8_16(p, v); }

// ---- math --------------------------------------------------------------------
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
// fast SiLU for the bf16/fp16 tensor-core paths (2-ulp exp and division)
__device__ __forceinline__ float siluf_(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// In-register unnormalised 32-point Walsh-Hadamard transform (Sylvester order:
// out[h] = sum_g (-1)^popc(g&h) in[g]).
__device__ __forceinline__ void fht32(float* v) {
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if ((i & s) == 0) {
        float a = v[i], b = v[i + s];
        v[i] = a + b;
        v[i + s] = a - b;
      }
    }
  }
}

// 2-bit ternary code (reference encoding: -1 -> 0b00, 0 -> 0b01, +1 -> 0b10),
// four values per byte, first value in the two most significant bits.
__device__ __forceinline__ float tern_val(uint32_t byte, int j) {
  return (float)((int)((byte >> (6 - 2 * j)) & 3u) - 1);
}

}  // namespace walsh

// ---- host-side argument checking ------------------------------------------------
#define WALSH_CHECK_ARG(cond) \
  do { if (!(cond)) return WALSH_ERR_ARG; } while (0)
#define WALSH_CHECK_SHAPE(cond) \
  do { if (!(cond)) return WALSH_ERR_SHAPE; } while (0)
#define WALSH_CHECK_DTYPE(d) \
  do { if ((d) != WALSH_F32 && (d) != WALSH_BF16 && (d) != WALSH_F16) return WALSH_ERR_DTYPE; } while (0)

// Calls F<T>(args...) with T the storage type of dtype code d.
#define WALSH_DISPATCH_DTYPE(d, T, ...)                        \
  [&]() -> int {                                               \
    if ((d) == WALSH_F32) { using T = float; return __VA_ARGS__; }         \
    if ((d) == WALSH_BF16) { using T = __nv_bfloat16; return __VA_ARGS__; } \
    { using T = __half; return __VA_ARGS__; }                  \
  }()

namespace walsh {
// Returns WALSH_ERR_INJECTED when the host-side fault injector is armed for
// `site` (environment variable WALSH_INJECT_FAULT=<site name> or "all").
int injected(const char* site);
// Converts the last launch error into a status code.
int launch_status();
}  // namespace walsh
