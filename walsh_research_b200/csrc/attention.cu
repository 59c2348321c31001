// Causal attention over the KV cache (CausalSelfAttention, src/model/chassis.py:442-466).
//
// Layouts: q [B, H, T, hd]; caches [B, H, ctx, hd]; o token-major [B, T, H, hd]
// so that the head mixer / wo kernels read whole token rows.  Query t sits at
// position start_pos + t and sees keys 0..start_pos+t (is_causal for the
// prompt, the tril(total-T) mask for cached steps).  Scores use exp2 with the
// 1/sqrt(hd) scale pre-multiplied by log2(e).
#include <math_constants.h>

#include <stdlib.h>
#include <type_traits>

#include "common.cuh"
#include "mma.cuh"

namespace walsh {

// Prefill: CTA = (64-query tile, head, batch); one thread per query, keys
// staged through shared memory 64 at a time.
template <int HD, typename T>
__global__ void __launch_bounds__(64)
attn_prefill_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc, int H, int Tq,
                    int ctx, int start_pos, float scale_log2, T* __restrict__ o) {
  constexpr int QT = 64, KT = 64;
  __shared__ float ks[KT][HD];
  __shared__ float vs[KT][HD];
  const int b = blockIdx.z, h = blockIdx.y, qt = blockIdx.x;
  const int t = qt * QT + threadIdx.x;
  const bool valid = t < Tq;
  const int qpos = start_pos + t;
  const size_t bh = (size_t)b * H + h;
  float qv[HD], acc[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    qv[d] = valid ? to_f(q[(bh * Tq + t) * HD + d]) * scale_log2 : 0.f;
    acc[d] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;
  const int kend = start_pos + min((qt + 1) * QT, Tq);  // one past the last key any query here sees
  const T* kb = kc + bh * ctx * HD;
  const T* vb = vc + bh * ctx * HD;
  for (int k0 = 0; k0 < kend; k0 += KT) {
    const int kn = min(KT, kend - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < KT * HD; i += QT) {
      const int j = i / HD, d = i - j * HD;
      const bool in = j < kn;
      ks[j][d] = in ? to_f(kb[(size_t)(k0 + j) * HD + d]) : 0.f;
      vs[j][d] = in ? to_f(vb[(size_t)(k0 + j) * HD + d]) : 0.f;
    }
    __syncthreads();
    float s[KT];
    float mt = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < HD; ++d) dot = fmaf(qv[d], ks[j][d], dot);
      s[j] = (j < kn && k0 + j <= qpos) ? dot : -CUDART_INF_F;
      mt = fmaxf(mt, s[j]);
    }
    const float mnew = fmaxf(m, mt);
    if (mnew == -CUDART_INF_F) continue;
    const float corr = exp2f(m - mnew);
    l *= corr;
#pragma unroll
    for (int d = 0; d < HD; ++d) acc[d] *= corr;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      const float p = exp2f(s[j] - mnew);
      l += p;
#pragma unroll
      for (int d = 0; d < HD; ++d) acc[d] = fmaf(p, vs[j][d], acc[d]);
    }
    m = mnew;
  }
  if (valid) {
    const float inv = 1.0f / l;
    T* op = o + (((size_t)b * Tq + t) * H + h) * HD;
#pragma unroll
    for (int d = 0; d < HD; ++d) op[d] = from_f<T>(acc[d] * inv);
  }
}

// Few queries (decode): CTA = (query, head, batch); 128 threads stride over
// the keys with private online-softmax state, merged through shared memory.
template <int HD, typename T>
__global__ void __launch_bounds__(128)
attn_decode_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc, int H, int Tq,
                   int ctx, int start_pos, float scale_log2, T* __restrict__ o) {
  constexpr int NT = 128;
  __shared__ float sm[NT], sl[NT];
  __shared__ float sacc[NT / 32][HD];
  const int b = blockIdx.z, h = blockIdx.y, t = blockIdx.x;
  const size_t bh = (size_t)b * H + h;
  const int nk = start_pos + t + 1;
  float qv[HD], acc[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    qv[d] = to_f(q[(bh * Tq + t) * HD + d]) * scale_log2;
    acc[d] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;
  const T* kb = kc + bh * ctx * HD;
  const T* vb = vc + bh * ctx * HD;
  for (int k = threadIdx.x; k < nk; k += NT) {
    float dot = 0.f;
#pragma unroll
    for (int d = 0; d < HD; ++d) dot = fmaf(qv[d], to_f(kb[(size_t)k * HD + d]), dot);
    const float mnew = fmaxf(m, dot);
    const float corr = exp2f(m - mnew);
    const float p = exp2f(dot - mnew);
    l = l * corr + p;
#pragma unroll
    for (int d = 0; d < HD; ++d) acc[d] = fmaf(p, to_f(vb[(size_t)k * HD + d]), acc[d] * corr);
    m = mnew;
  }
  sm[threadIdx.x] = m;
  __syncthreads();
  float M = -CUDART_INF_F;
  for (int i = 0; i < NT; ++i) M = fmaxf(M, sm[i]);
  const float f = (m == -CUDART_INF_F) ? 0.f : exp2f(m - M);
  sl[threadIdx.x] = l * f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    const float v = warp_sum(acc[d] * f);
    if (lane == 0) sacc[warp][d] = v;
  }
  __syncthreads();
  if (threadIdx.x < HD) {
    float L = 0.f;
    for (int i = 0; i < NT; ++i) L += sl[i];
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) v += sacc[w][threadIdx.x];
    o[(((size_t)b * Tq + t) * H + h) * HD + threadIdx.x] = from_f<T>(v / L);
  }
}

// ---------------------------------------------------------------------------
// Decode attention for 16-bit caches (the batched decode step: one or a few
// new queries against a long cache).  Pure KV streaming, so the kernel is
// built for HBM bandwidth: CTA = one query of one (batch, head); LPK = HD/8
// lanes share one key row, each lane loading one 16-byte vector of K and of
// V, so a warp-wide load covers 32/LPK whole rows (512 contiguous bytes);
// every thread issues the loads of KPT keys before using any of them; an
// online softmax (exp2 domain) runs per chunk of KPT keys; the per-thread
// (max, sum, acc) triples are merged across lanes with shuffles and across
// warps through shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void merge_parts(float& m, float& l, float* acc, float m2, float l2, const float* acc2) {
  const float mn = fmaxf(m, m2);
  const float f1 = mn == -CUDART_INF_F ? 0.f : ex2_f32(m - mn);
  const float f2 = mn == -CUDART_INF_F ? 0.f : ex2_f32(m2 - mn);
  l = l * f1 + l2 * f2;
#pragma unroll
  for (int d = 0; d < 8; ++d) acc[d] = acc[d] * f1 + acc2[d] * f2;
  m = mn;
}

template <int HD, typename T>
__global__ void __launch_bounds__(128)
attn_decode_vec_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc, int H, int Tq,
                       int ctx, int start_pos, float scale_log2, T* __restrict__ o) {
  constexpr int NT = 128, NW = NT / 32, LPK = HD / 8, KPT = 8;
  constexpr int SLOTS = NT / LPK;  // keys in flight per load step of the CTA
  __shared__ float red[NW][LPK][10];
  const int b = blockIdx.z, h = blockIdx.y, t = blockIdx.x;
  const size_t bh = (size_t)b * H + h;
  const int nk = start_pos + t + 1;  // keys visible to this query
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sub = lane % LPK, slot = tid / LPK;
  float qv[8];
  load8(q + (bh * Tq + t) * HD + sub * 8, qv);
#pragma unroll
  for (int d = 0; d < 8; ++d) qv[d] *= scale_log2;
  const uint4* kb = reinterpret_cast<const uint4*>(kc + bh * (size_t)ctx * HD) + sub;
  const uint4* vb = reinterpret_cast<const uint4*>(vc + bh * (size_t)ctx * HD) + sub;
  float m = -CUDART_INF_F, l = 0.f, acc[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) acc[d] = 0.f;
  // the trip count is the same for every thread (the dot shuffles need the whole warp)
  for (int c0 = 0; c0 < nk; c0 += SLOTS * KPT) {
    const int k0 = c0 + slot;
    uint4 kr[KPT], vr[KPT];
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const int k = k0 + i * SLOTS;
      if (k < nk) {
        kr[i] = __ldg(kb + (size_t)k * LPK);
        vr[i] = __ldg(vb + (size_t)k * LPK);
      } else {
        kr[i] = vr[i] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float s[KPT];
    float cm = -CUDART_INF_F;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      float kv[8];
      unpack8(kr[i], kv, (const T*)nullptr);
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < 8; ++d) dot = fmaf(qv[d], kv[d], dot);
#pragma unroll
      for (int off = 1; off < LPK; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      s[i] = (k0 + i * SLOTS < nk) ? dot : -CUDART_INF_F;
      cm = fmaxf(cm, s[i]);
    }
    const float mn = fmaxf(m, cm);  // -inf only while this thread has seen no visible key
    const float corr = mn == -CUDART_INF_F ? 1.f : ex2_f32(m - mn);
    const float sub_m = mn == -CUDART_INF_F ? 0.f : mn;
    l *= corr;
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[d] *= corr;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const float p = ex2_f32(s[i] - sub_m);  // masked keys: 2^-inf = 0
      float vv[8];
      unpack8(vr[i], vv, (const T*)nullptr);
      l += p;
#pragma unroll
      for (int d = 0; d < 8; ++d) acc[d] = fmaf(p, vv[d], acc[d]);
    }
    m = mn;
  }
  // lanes of the same channel group hold disjoint key sets: merge them
#pragma unroll
  for (int off = LPK; off < 32; off <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off), l2 = __shfl_xor_sync(0xffffffffu, l, off);
    float a2[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) a2[d] = __shfl_xor_sync(0xffffffffu, acc[d], off);
    merge_parts(m, l, acc, m2, l2, a2);
  }
  if (lane < LPK) {
    red[warp][sub][0] = m;
    red[warp][sub][1] = l;
#pragma unroll
    for (int d = 0; d < 8; ++d) red[warp][sub][2 + d] = acc[d];
  }
  __syncthreads();
  if (tid < LPK) {
#pragma unroll
    for (int w = 1; w < NW; ++w) merge_parts(m, l, acc, red[w][sub][0], red[w][sub][1], &red[w][sub][2]);
    const float inv = 1.0f / l;
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[d] *= inv;
    store8(o + (((size_t)b * Tq + t) * H + h) * HD + sub * 8, acc);
  }
}

// ---------------------------------------------------------------------------
// bf16 prefill on the tensor cores (flash-attention dataflow with mma.sync):
// CTA = 128 queries of one (batch, head), 8 warps x 16 query rows; K/V tiles
// of 64 keys double-buffered in shared memory by cp.async; S = Q K^T and
// O += P V with m16n8k16 bf16 MMAs (fp32 accumulate), the S accumulators
// re-packed in registers as the A operand of P V; online softmax in exp2.
// ---------------------------------------------------------------------------
template <int HD, typename TE, int KT>
__global__ void __launch_bounds__(256)
attn_mma_kernel(const TE* __restrict__ q, const TE* __restrict__ kc, const TE* __restrict__ vc, int H, int Tq,
                int ctx, int start_pos, float scale_log2, TE* __restrict__ o) {
  constexpr int QT = 128, LD = HD + 8;  // padded rows: conflict-free ldmatrix
  constexpr int CH = HD / 8;                     // 16-byte chunks per row
  __shared__ __align__(16) TE Qs[QT][LD];
  __shared__ __align__(16) TE Ks[2][KT][LD];
  __shared__ __align__(16) TE Vs[2][KT][LD];
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = (gridDim.x - 1 - blockIdx.x) * QT;  // longest (latest) query tiles first
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const size_t bh = (size_t)b * H + h;
  const TE* qb = q + bh * Tq * HD;
  const TE* kb = kc + bh * ctx * HD;
  const TE* vb = vc + bh * ctx * HD;
  const int kend = start_pos + min(q0 + QT, Tq);  // keys [0, kend) are visible to some query here
  const int nkt = (kend + KT - 1) / KT;

  for (int i = tid; i < QT * CH; i += 256) {
    const int r = i / CH, c = i - r * CH;
    const bool in = q0 + r < Tq;
    cp_async16(&Qs[r][c * 8], qb + (size_t)(in ? q0 + r : 0) * HD + c * 8, in ? 16 : 0);
  }
  auto load_kv = [&](int kt, int buf) {
    for (int i = tid; i < 2 * KT * CH; i += 256) {
      const int which = i / (KT * CH), j = i - which * KT * CH;
      const int r = j / CH, c = j - r * CH;
      const int key = kt * KT + r;
      const bool in = key < kend;
      const TE* src = (which ? vb : kb) + (size_t)(in ? key : 0) * HD + c * 8;
      cp_async16(which ? &Vs[buf][r][c * 8] : &Ks[buf][r][c * 8], src, in ? 16 : 0);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const int qrow0 = warp * 16;
  const int qp_lo = start_pos + q0 + qrow0 + g;  // query positions of this thread's two rows
  const int qp_hi = qp_lo + 8;
  const int qp_warp_max = start_pos + q0 + qrow0 + 15;
  float m_lo = -CUDART_INF_F, m_hi = -CUDART_INF_F, l_lo = 0.f, l_hi = 0.f;
  float oacc[HD / 8 + 1][4];  // last n-tile: P row sums (fp16 path)
#pragma unroll
  for (int i = 0; i < HD / 8 + 1; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
  uint32_t qf[HD / 16][4];

  for (int kt = 0; kt < nkt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nkt) load_kv(kt + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks)
        ldsm_x4(qf[ks], &Qs[qrow0 + (lane & 15)][ks * 16 + (lane >> 4) * 8]);
    }
    if (kt * KT <= qp_warp_max) {  // some key of this tile is visible to this warp's rows
      float s[KT / 8][4];
#pragma unroll
      for (int n = 0; n < KT / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks)
#pragma unroll
        for (int np = 0; np < KT / 16; ++np) {
          uint32_t kf[4];
          ldsm_x4(kf, &Ks[buf][np * 16 + (lane & 7) + ((lane >> 4) << 3)][ks * 16 + ((lane >> 3) & 1) * 8]);
          mma16<TE>(s[2 * np], qf[ks], kf[0], kf[1]);
          mma16<TE>(s[2 * np + 1], qf[ks], kf[2], kf[3]);
        }
      const bool diag = (kt + 1) * KT - 1 > start_pos + q0 + qrow0;  // tile may hold masked keys
      // row maxima of the raw scores (masked entries -inf)
      float mt_lo = -CUDART_INF_F, mt_hi = -CUDART_INF_F;
#pragma unroll
      for (int n = 0; n < KT / 8; ++n) {
        const int key = kt * KT + n * 8 + 2 * t4;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (diag) {
            if (key + e > qp_lo) s[n][e] = -CUDART_INF_F;
            if (key + e > qp_hi) s[n][2 + e] = -CUDART_INF_F;
          }
          mt_lo = fmaxf(mt_lo, s[n][e]);
          mt_hi = fmaxf(mt_hi, s[n][2 + e]);
        }
      }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mt_lo = fmaxf(mt_lo, __shfl_xor_sync(0xffffffffu, mt_lo, off));
        mt_hi = fmaxf(mt_hi, __shfl_xor_sync(0xffffffffu, mt_hi, off));
      }
      const float mn_lo = fmaxf(m_lo, mt_lo), mn_hi = fmaxf(m_hi, mt_hi);
      // rows with no visible key yet keep m = -inf; subtract 0 so exp2 gives 0, not NaN
      const float sub_lo = mn_lo == -CUDART_INF_F ? 0.f : mn_lo * scale_log2;
      const float sub_hi = mn_hi == -CUDART_INF_F ? 0.f : mn_hi * scale_log2;
      // the O / row-sum rescale is skipped when no row maximum of this warp moved
      const bool moved = __any_sync(0xffffffffu, mn_lo != m_lo || mn_hi != m_hi);
      const float corr_lo = moved ? ex2_f32(m_lo * scale_log2 - sub_lo) : 1.f;
      const float corr_hi = moved ? ex2_f32(m_hi * scale_log2 - sub_hi) : 1.f;
      m_lo = mn_lo;
      m_hi = mn_hi;
      uint32_t pf[KT / 16][4];
      if constexpr (std::is_same<TE, __half>::value) {
        // p = 2^(s * scale - m * scale) two at a time in fp16 (the P V operand precision)
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
          pf[n >> 1][(n & 1) * 2 + 0] =
              ex2_f16x2(pack_f16(fmaf(s[n][0], scale_log2, -sub_lo), fmaf(s[n][1], scale_log2, -sub_lo)));
          pf[n >> 1][(n & 1) * 2 + 1] =
              ex2_f16x2(pack_f16(fmaf(s[n][2], scale_log2, -sub_hi), fmaf(s[n][3], scale_log2, -sub_hi)));
        }
      } else {
        float rs_lo = 0.f, rs_hi = 0.f;
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
          const float p0 = exp2f(fmaf(s[n][0], scale_log2, -sub_lo)), p1 = exp2f(fmaf(s[n][1], scale_log2, -sub_lo));
          const float p2 = exp2f(fmaf(s[n][2], scale_log2, -sub_hi)), p3 = exp2f(fmaf(s[n][3], scale_log2, -sub_hi));
          rs_lo += p0 + p1;
          rs_hi += p2 + p3;
          pf[n >> 1][(n & 1) * 2 + 0] = pack2<TE>(p0, p1);
          pf[n >> 1][(n & 1) * 2 + 1] = pack2<TE>(p2, p3);
        }
        l_lo = l_lo * corr_lo + rs_lo;
        l_hi = l_hi * corr_hi + rs_hi;
      }
      if (moved) {
#pragma unroll
        for (int i = 0; i < HD / 8 + 1; ++i) {
          oacc[i][0] *= corr_lo; oacc[i][1] *= corr_lo;
          oacc[i][2] *= corr_hi; oacc[i][3] *= corr_hi;
        }
      }
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk) {
        // A operand = P[16 rows][16 keys]: registers {tile 2kk (c0c1), tile 2kk (c2c3), tile 2kk+1 (c0c1), tile 2kk+1 (c2c3)}
        const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
        for (int dp = 0; dp < HD / 16; ++dp) {
          uint32_t vf[4];
          ldsm_x4_t(vf, &Vs[buf][kk * 16 + (lane & 15)][dp * 16 + (lane >> 4) * 8]);
          mma16<TE>(oacc[2 * dp], a, vf[0], vf[1]);
          mma16<TE>(oacc[2 * dp + 1], a, vf[2], vf[3]);
        }
        if constexpr (std::is_same<TE, __half>::value)  // row sums of P on the tensor cores (V column of ones)
          mma16<TE>(oacc[HD / 8], a, 0x3C003C00u, 0x3C003C00u);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }
  if constexpr (std::is_same<TE, __half>::value) {
    l_lo = oacc[HD / 8][0];
    l_hi = oacc[HD / 8][2];
  } else {
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
      l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
    }
  }
  const float inv_lo = 1.0f / l_lo, inv_hi = 1.0f / l_hi;
  const int t_lo = q0 + qrow0 + g, t_hi = t_lo + 8;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int d = i * 8 + 2 * t4;
    if (t_lo < Tq)
      *reinterpret_cast<uint32_t*>(o + (((size_t)b * Tq + t_lo) * H + h) * HD + d) =
          pack2<TE>(oacc[i][0] * inv_lo, oacc[i][1] * inv_lo);
    if (t_hi < Tq)
      *reinterpret_cast<uint32_t*>(o + (((size_t)b * Tq + t_hi) * H + h) * HD + d) =
          pack2<TE>(oacc[i][2] * inv_hi, oacc[i][3] * inv_hi);
  }
}

// ---------------------------------------------------------------------------
// fp16 prefill, hd 16, whole-head variant: one CTA per (batch, head) holds
// that head's visible K and V (up to 2048 keys, rows padded to 48 bytes for
// conflict-free ldmatrix) in shared memory, loaded once with cp.async; the 8
// warps then run 16-row query tiles independently (no barriers), tiles
// dealt out snake-wise (w, 15 - w, 16 + w, ...) so every warp gets the same
// causal work.  Per 64-key step: S - m = Q K^T - m (8 MMAs whose addend is
// the row's reference maximum), row maxima, P = 2^(S - m) as paired fp16
// ex2, O += P V and the row sums of P (all-ones V column) on the tensor
// cores.  The reference maximum m of a row only moves when the row maximum
// exceeds it by more than 8 (P <= 256 in fp16), so the O rescale (and the
// explicit subtraction of the shift) is rare.
// ---------------------------------------------------------------------------
constexpr int kAttnHeadMaxKeys = 2048;
// Bit n set: exponent pairs of n-tile n (of the 8 per 64-key step) are
// evaluated by the FMA-pipe polynomial instead of MUFU ex2.  Measured on
// B200 at B64 x H32 x T1024: 421 us with none, 458 us with 2 of 8, 481 us
// with 3 of 8, 495 us with 4 of 8 -- with Q pre-scaled and three-input
// maxima the MUFU pipe no longer bounds this kernel, so the default is none.
#ifndef WALSH_ATTN_POLY_PAIRS
#define WALSH_ATTN_POLY_PAIRS 0x00
#endif

// Byte offset of 16-byte half c (0, 1) of key row r in a K or V tile of
// 32-byte rows: the halves trade places on every other group of four rows,
// so the eight rows one ldmatrix phase reads (one half each) fall in eight
// distinct bank quads, with and without .trans.
__device__ __forceinline__ uint32_t kv_swz(int r, int c) {
  return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
}

// 64 KB of K and V at 1024 keys: three CTAs (24 warps) per SM.
// F32P: P = 2^(S - m) as f32 exponentials whose row sums are packed f32x2
// adds on the FMA pipe, P rounded to fp16 only as the P V operand (16 legacy
// MMAs per 1024 scores); otherwise paired fp16 exponentials with the row sums
// as an all-ones MMA column (20 MMAs).
template <bool F32P>
__global__ void __launch_bounds__(256, 3)
attn_head_kernel(const __half* __restrict__ q, const __half* __restrict__ kc, const __half* __restrict__ vc, int H,
                 int Tq, int ctx, int start_pos, float scale_log2, __half* __restrict__ o) {
  constexpr int HD = 16, KT = 64;
  extern __shared__ __align__(16) unsigned char smb[];
  unsigned char* Ks = smb;  // [kpad] rows of 32 bytes (kv_swz)
  const int b = blockIdx.y, h = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const size_t bh = (size_t)b * H + h;
  const int kend = start_pos + Tq;
  const int kpad = (kend + KT - 1) / KT * KT;  // the last 64-key step reads up to here
  unsigned char* Vs = smb + (size_t)kpad * 32;  // [kpad] rows of 32 bytes (kv_swz)
  const __half* kb = kc + bh * ctx * HD;
  const __half* vb = vc + bh * ctx * HD;
  for (int i = tid; i < kpad * 2; i += 256) {
    const int r = i >> 1, c = i & 1;
    const bool in = r < kend;  // rows kend..kpad-1 are zero-filled
    cp_async16(Ks + kv_swz(r, c), kb + (size_t)(in ? r : 0) * HD + c * 8, in ? 16 : 0);
    cp_async16(Vs + kv_swz(r, c), vb + (size_t)(in ? r : 0) * HD + c * 8, in ? 16 : 0);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // this lane's ldmatrix row addresses within a 16-key group (the group
  // start is a multiple of 8 rows, so the swizzle depends on the lane only)
  const uint32_t k_lane = kv_swz((lane & 7) + ((lane >> 4) << 3), (lane >> 3) & 1);
  const uint32_t v_lane = kv_swz(lane & 15, lane >> 4);

  const __half* qb = q + bh * Tq * HD;
  const int nqt = (Tq + 15) / 16;
  for (int i = 0;; ++i) {
    const int qt = i * 8 + ((i & 1) ? 7 - warp : warp);
    if (qt >= nqt) break;
    const int q0 = qt * 16;
    const int r_lo = q0 + g, r_hi = r_lo + 8;
    // Q fragment straight from global memory (rows past Tq are zero)
    uint32_t qf[4];
    {
      const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qb);
      qf[0] = r_lo < Tq ? __ldg(q32 + (r_lo * HD + 2 * t4) / 2) : 0u;
      qf[1] = r_hi < Tq ? __ldg(q32 + (r_hi * HD + 2 * t4) / 2) : 0u;
      qf[2] = r_lo < Tq ? __ldg(q32 + (r_lo * HD + 2 * t4 + 8) / 2) : 0u;
      qf[3] = r_hi < Tq ? __ldg(q32 + (r_hi * HD + 2 * t4 + 8) / 2) : 0u;
      // fold the softmax scale (and log2 e) into Q: S comes out in the exp2 domain
      const __half2 sc = __float2half2_rn(scale_log2);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half2 v;
        memcpy(&v, &qf[j], 4);
        v = __hmul2(v, sc);
        memcpy(&qf[j], &v, 4);
      }
    }
    const int qp_lo = start_pos + r_lo, qp_hi = start_pos + r_hi;  // query positions
    const int nkey = min(kend, start_pos + q0 + 16);                // keys visible to some row
    // reference maxima (exp2 domain): 0 until a row sees its first key; the MMA
    // starts from -m, so S - m comes out of the tensor core
    float m_lo = 0.f, m_hi = 0.f;
    // a row's reference maximum moves once its row maximum passes m + thr:
    // thr = -inf until the row's first visible key, 8 after (P <= 256 in fp16)
    float thr_lo = -CUDART_INF_F, thr_hi = -CUDART_INF_F;
    float oacc[HD / 8 + 1][4];
#pragma unroll
    for (int j = 0; j < HD / 8 + 1; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
    uint64_t l2_lo = 0, l2_hi = 0;  // F32P: this thread's partial row sums (column pairs)
    for (int k0 = 0; k0 < nkey; k0 += KT) {
      float s[KT / 8][4];
#pragma unroll
      for (int np = 0; np < KT / 16; ++np) {
        uint32_t kf[4];
        ldsm_x4(kf, Ks + k_lane + (k0 + np * 16) * 32);
        mma_f16_rowc(s[2 * np], qf, kf[0], kf[1], -m_lo, -m_hi);
        mma_f16_rowc(s[2 * np + 1], qf, kf[2], kf[3], -m_lo, -m_hi);
      }
      // keys past a row's position (or past kend) are masked
      const bool edge = k0 + KT > start_pos + q0 || k0 + KT > kend;
      if (edge) {
#pragma unroll
        for (int n = 0; n < KT / 8; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = k0 + n * 8 + 2 * t4 + e;
            if (key > qp_lo || key >= kend) s[n][e] = -CUDART_INF_F;
            if (key > qp_hi || key >= kend) s[n][2 + e] = -CUDART_INF_F;
          }
      }
      // row maxima of S - m
      float mt_lo = -CUDART_INF_F, mt_hi = -CUDART_INF_F;
#pragma unroll
      for (int n = 0; n < KT / 8; ++n) {
        mt_lo = fmax3(mt_lo, s[n][0], s[n][1]);
        mt_hi = fmax3(mt_hi, s[n][2], s[n][3]);
      }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mt_lo = fmaxf(mt_lo, __shfl_xor_sync(0xffffffffu, mt_lo, off));
        mt_hi = fmaxf(mt_hi, __shfl_xor_sync(0xffffffffu, mt_hi, off));
      }
      const bool mv_lo = mt_lo > thr_lo, mv_hi = mt_hi > thr_hi;
      if (__any_sync(0xffffffffu, mv_lo || mv_hi)) {
        // move m by d = the step's row maximum: O *= 2^-d, this step's S - m -= d
        // (before a row's first key O is zero and stays so: factor 0, as 2^-d may overflow)
        const float d_lo = mv_lo ? mt_lo : 0.f, d_hi = mv_hi ? mt_hi : 0.f;
        const float c_lo = thr_lo == -CUDART_INF_F ? 0.f : ex2_f32(-d_lo);
        const float c_hi = thr_hi == -CUDART_INF_F ? 0.f : ex2_f32(-d_hi);
#pragma unroll
        for (int j = 0; j < HD / 8 + 1; ++j) {
          oacc[j][0] *= c_lo; oacc[j][1] *= c_lo;
          oacc[j][2] *= c_hi; oacc[j][3] *= c_hi;
        }
        if (F32P) {
          l2_lo = f2_mul(l2_lo, f2_dup(c_lo));
          l2_hi = f2_mul(l2_hi, f2_dup(c_hi));
        }
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
          s[n][0] -= d_lo; s[n][1] -= d_lo;
          s[n][2] -= d_hi; s[n][3] -= d_hi;
        }
        m_lo += d_lo;
        m_hi += d_hi;
        if (mv_lo) thr_lo = 8.f;
        if (mv_hi) thr_hi = 8.f;
      }
      // P = 2^(S - m) (rows with no visible key yet: 2^-inf = 0): the pairs selected
      // by WALSH_ATTN_POLY_PAIRS on the FMA pipe, the rest as paired fp16 ex2 on
      // the MUFU pipe
      uint32_t pf[KT / 16][4];
      if (F32P) {
        const uint64_t one2 = f2_dup(1.f);
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
          const float p0 = ex2_f32(s[n][0]), p1 = ex2_f32(s[n][1]), p2 = ex2_f32(s[n][2]), p3 = ex2_f32(s[n][3]);
          pf[n >> 1][(n & 1) * 2 + 0] = pack_f16(p0, p1);
          pf[n >> 1][(n & 1) * 2 + 1] = pack_f16(p2, p3);
          l2_lo = f2_fma(f2_pack(p0, p1), one2, l2_lo);
          l2_hi = f2_fma(f2_pack(p2, p3), one2, l2_hi);
        }
      } else {
#pragma unroll
      for (int n = 0; n < KT / 8; ++n) {
        if ((WALSH_ATTN_POLY_PAIRS >> n) & 1) {
          pf[n >> 1][(n & 1) * 2 + 0] = pack_f16(exp2_poly(s[n][0]), exp2_poly(s[n][1]));
          pf[n >> 1][(n & 1) * 2 + 1] = pack_f16(exp2_poly(s[n][2]), exp2_poly(s[n][3]));
        } else {
          pf[n >> 1][(n & 1) * 2 + 0] = ex2_f16x2(pack_f16(s[n][0], s[n][1]));
          pf[n >> 1][(n & 1) * 2 + 1] = ex2_f16x2(pack_f16(s[n][2], s[n][3]));
        }
      }
      }
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk) {
        uint32_t vf[4];
        ldsm_x4_t(vf, Vs + v_lane + (k0 + kk * 16) * 32);
        mma_f16(oacc[0], pf[kk], vf[0], vf[1]);
        mma_f16(oacc[1], pf[kk], vf[2], vf[3]);
        if (!F32P) mma_f16(oacc[HD / 8], pf[kk], 0x3C003C00u, 0x3C003C00u);  // row sums of P
      }
    }
    float l_lo, l_hi;
    if (F32P) {  // the quad's four threads hold the row's column pairs
      l_lo = __uint_as_float((uint32_t)l2_lo) + __uint_as_float((uint32_t)(l2_lo >> 32));
      l_hi = __uint_as_float((uint32_t)l2_hi) + __uint_as_float((uint32_t)(l2_hi >> 32));
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
        l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
      }
    } else {
      l_lo = oacc[HD / 8][0];
      l_hi = oacc[HD / 8][2];
    }
    const float inv_lo = 1.0f / l_lo, inv_hi = 1.0f / l_hi;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      const int d = j * 8 + 2 * t4;
      if (r_lo < Tq)
        *reinterpret_cast<uint32_t*>(o + (((size_t)b * Tq + r_lo) * H + h) * HD + d) =
            pack_f16_sat(oacc[j][0] * inv_lo, oacc[j][1] * inv_lo);
      if (r_hi < Tq)
        *reinterpret_cast<uint32_t*>(o + (((size_t)b * Tq + r_hi) * H + h) * HD + d) =
            pack_f16_sat(oacc[j][2] * inv_hi, oacc[j][3] * inv_hi);
    }
  }
}

// tcgen05 prefill kernel (attention_tc.cu): 1 when it ran, 0 when it does not apply
int launch_attn_tc05(const void* q, const void* kc, const void* vc, int B, int H, int Tq, int ctx, int start_pos,
                     float scale_log2, void* o, cudaStream_t s);

template <int HD, typename T>
static int launch_attn(const void* q, const void* kc, const void* vc, int B, int H, int Tq, int ctx,
                       int start_pos, void* o, cudaStream_t s) {
  const float scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
  const bool aligned = ((((uintptr_t)q) | ((uintptr_t)kc) | ((uintptr_t)vc)) & 15u) == 0;
  if constexpr (std::is_same<T, __half>::value && HD == 16) {
    if (const int r = launch_attn_tc05(q, kc, vc, B, H, Tq, ctx, start_pos, scale_log2, o, s)) return r < 0 ? r : WALSH_OK;
    const int kend = start_pos + Tq;
    if (Tq > 4 && aligned && kend <= kAttnHeadMaxKeys && H <= 65535 && B <= 65535) {
      const int smem = 2 * ((kend + 63) / 64 * 64) * HD * (int)sizeof(__half);
      // f32 exponentials + FMA-pipe row sums: 361 us at B64 x H32 x T1024
      // against 382 us for the paired fp16 form with the all-ones MMA column
      auto* kern = attn_head_kernel<true>;
      if (smem > 48 * 1024 &&
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return launch_status();
      kern<<<dim3(H, B), 256, smem, s>>>((const __half*)q, (const __half*)kc, (const __half*)vc, H, Tq,
                                                     ctx, start_pos, scale_log2, (__half*)o);
      return launch_status();
    }
  }
  if constexpr (sizeof(T) == 2) {
    if (Tq > 4 && aligned) {
      dim3 grid((Tq + 127) / 128, H, B);
      attn_mma_kernel<HD, T, 64><<<grid, 256, 0, s>>>((const T*)q, (const T*)kc, (const T*)vc, H, Tq, ctx,
                                                       start_pos, scale_log2, (T*)o);
      return launch_status();
    }
  }
  if constexpr (sizeof(T) == 2) {
    if (Tq <= 4 && aligned && (((uintptr_t)o) & 15u) == 0) {
      dim3 grid(Tq, H, B);
      attn_decode_vec_kernel<HD, T><<<grid, 128, 0, s>>>((const T*)q, (const T*)kc, (const T*)vc, H, Tq, ctx,
                                                        start_pos, scale_log2, (T*)o);
      return launch_status();
    }
  }
  if (Tq <= 4) {
    dim3 grid(Tq, H, B);
    attn_decode_kernel<HD, T><<<grid, 128, 0, s>>>((const T*)q, (const T*)kc, (const T*)vc, H, Tq, ctx,
                                                  start_pos, scale_log2, (T*)o);
  } else {
    dim3 grid((Tq + 63) / 64, H, B);
    attn_prefill_kernel<HD, T><<<grid, 64, 0, s>>>((const T*)q, (const T*)kc, (const T*)vc, H, Tq, ctx,
                                                  start_pos, scale_log2, (T*)o);
  }
  return launch_status();
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_attn_fwd(const void* q, const void* k_cache, const void* v_cache, int dtype,
                                       int B, int H, int T, int hd, int ctx, int start_pos, void* o,
                                       void* stream) {
  if (int e = injected("attn_fwd")) return e;
  WALSH_CHECK_DTYPE(dtype);
  WALSH_CHECK_ARG(q && k_cache && v_cache && o);
  WALSH_CHECK_SHAPE(B > 0 && H > 0 && T > 0 && start_pos >= 0 && start_pos + T <= ctx);
  WALSH_CHECK_SHAPE(B <= 65535 && H <= 65535);
  cudaStream_t s = (cudaStream_t)stream;
  if (hd != 16 && hd != 32) return WALSH_ERR_SHAPE;
  return WALSH_DISPATCH_DTYPE(dtype, ET, hd == 16 ? launch_attn<16, ET>(q, k_cache, v_cache, B, H, T, ctx, start_pos, o, s)
                                                  : launch_attn<32, ET>(q, k_cache, v_cache, B, H, T, ctx, start_pos, o, s));
}
