// Causal prefill attention, head dim 16, fp16, on the 5th-generation tensor
// cores (sm_100a): S = Q K^T and O = P V as tcgen05 MMAs with fp32
// accumulators in tensor memory.
//
// Work split: a CTA takes one (batch, head) and half of its 128-row query
// tiles, paired first/last (tiles t and n-1-t carry causal work n together),
// so both CTAs of a head get the same number of 64-key steps.  Each CTA
// stages, once, its head's keys and values and its query tiles in shared
// memory in the 128-byte-swizzled K-major layout the MMA reads:
//  - K (head dim 16 = 32 bytes a row) four key blocks side by side in one
//    128-byte row: block j is the k-slice j % 4 of a 64-row tile, and the
//    S MMA of block j reads it with the descriptor advanced by 32 (j % 4)
//    bytes -- one MMA (M 128, N 64, K 16) per 64-key step;
//  - the query tiles of the CTA (at most four) the same way in one 128-row tile;
//  - V transposed (16 dims x 64 keys per block, the B operand of P V);
//  - a 16 x 64 tile of ones: P . ones = the row sums of P on the tensor core.
// Warps 0-3 each own one tensor-memory lane quarter = 32 query rows: a thread
// reads its row of S (64 fp32 values) with tcgen05.ld, so row maxima need no
// shuffles, and writes its row of P = 2^(S scale - m) (paired fp16 ex2) back
// into tensor memory with tcgen05.st, where the P V MMA reads it as its A
// operand.  Warp 4 allocates tensor memory and one of its threads issues the
// MMAs.  S and P are double-buffered in tensor memory, so the MMAs of step
// g + 1 run while the threads work on step g.  The reference maximum m of a
// row moves only when its row maximum passes m + 8 (P <= 256 in fp16); then
// the thread rescales its O and row-sum accumulators in tensor memory after
// the previous P V step has completed.
//
// Every wait on an mbarrier is bounded; a wait that runs out marks the CTA
// aborted, every role leaves its loop, tensor memory is freed and
// g_attn_tc05_error records WALSH_ERR_TIMEOUT.
//
// Replaces the prefill scaled_dot_product_attention call of
// CausalSelfAttention.forward (src/model/chassis.py:442-466).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>
#include <stdlib.h>

#include "common.cuh"
#include "mma.cuh"
#include "tc05.cuh"

// probe hook (slot, step): no code unless a profiling build defines it
#ifndef ATTN_TC_TRACE
#define ATTN_TC_TRACE(slot, step)
#endif

namespace walsh {
namespace attn_tc {

constexpr int NSOFT = 8;           // softmax warps: two warpgroups on different query tiles
constexpr int MMA_WARP = NSOFT;    // TMEM allocation + MMA issue
constexpr int NTHREADS = 32 * (NSOFT + 1);
constexpr int MAX_KEYS = 1024;     // keys a CTA holds in shared memory
constexpr int MAX_QTILES = 8;      // 128-row query tiles per head (4 per CTA)
constexpr int TILE_BYTES = 128 * 128;      // 128 rows x 128 bytes
constexpr int KSUPER_BYTES = 64 * 128;     // 64 rows x 128 bytes = 4 key blocks
constexpr int VT_BLOCK_BYTES = 16 * 128;   // 16 dims x 64 keys
constexpr int ONES_BYTES = 16 * 128;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t WG_COLS = 128;  // tensor-memory columns of one softmax warpgroup:
constexpr uint32_t COL_S = 0;      //   64 fp32 S
constexpr uint32_t COL_P = 64;     //   32 columns of P (fp16 pairs)
constexpr uint32_t COL_O = 96;     //   16 columns of O
constexpr uint32_t COL_SUM = 112;  //   16 columns, all equal to the row sum
constexpr float kMasked = -1.0e6f;  // score of a masked key (finite: see exp2_pair_fma)
constexpr int SMEM_FLOOR = 80 * 1024;  // at most two CTAs (2 x 256 TMEM columns) per SM

// shared-memory byte offsets from the 1024-aligned base
constexpr int OFF_Q = 0;
constexpr int OFF_ONES = OFF_Q + TILE_BYTES;
constexpr int OFF_K = OFF_ONES + 1024 * ((ONES_BYTES + 1023) / 1024);  // 1024-aligned

__host__ __device__ inline int vt_offset(int nkb) { return OFF_K + (nkb + 3) / 4 * KSUPER_BYTES; }
__host__ __device__ inline int bar_offset(int nkb) { return vt_offset(nkb) + nkb * VT_BLOCK_BYTES; }
__host__ inline int smem_bytes(int nkb) {
  const int b = 1024 + bar_offset(nkb) + 128;
  return b < SMEM_FLOOR ? SMEM_FLOOR : b;
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `r` in a 128B-swizzled tile
__device__ __forceinline__ uint32_t sw_off(int r, int chunk) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4));
}

// 64-key blocks that query tile t needs
__device__ __forceinline__ int tile_blocks(int t, int start_pos, int kend) {
  return (min(kend, start_pos + 128 * t + 128) + 63) >> 6;
}

// warpgroup owning entry i of a CTA's tile list: with 3-4 tiles the first pair
// (or the first two) go to warpgroup 0, the rest to 1; with 1-2 one tile each
__device__ __forceinline__ int tile_owner(int i, int ntile) { return ntile >= 3 ? (i >= 2) : i; }

// the query tiles of CTA half `half`: pairs (p, n-1-p) with p = half, half+2, ...
__device__ __forceinline__ int cta_tiles(int half, int nqt, int* tiles) {
  int n = 0;
  for (int p = half; 2 * p <= nqt - 1; p += 2) {
    tiles[n++] = p;
    if (p < nqt - 1 - p) tiles[n++] = nqt - 1 - p;
  }
  return n;
}


__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from registers
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns from registers
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// D[tmem] (+)= A[tmem] . B[smem]^T (A: M rows in lanes, K fp16 two per column), one thread
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// (a, b) * (s, s) + (c, c) as one packed fp32 FMA
__device__ __forceinline__ float2 ffma2(float a, float b, float s, float c) {
  uint64_t r;
  const uint64_t x = ((uint64_t)__float_as_uint(b) << 32) | __float_as_uint(a);
  const uint64_t y = ((uint64_t)__float_as_uint(s) << 32) | __float_as_uint(s);
  const uint64_t z = ((uint64_t)__float_as_uint(c) << 32) | __float_as_uint(c);
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(x), "l"(y), "l"(z));
  return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}

__device__ __forceinline__ uint64_t pk2(float v) {
  return ((uint64_t)__float_as_uint(v) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t x, uint64_t y) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(x), "l"(y));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t x, uint64_t y, uint64_t z) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(x), "l"(y), "l"(z));
  return r;
}

constexpr float kShift = 12582912.f;  // 1.5 * 2^23: adding it rounds to an integer

// P = 2^(s scale - m) for two scores as packed fp16, entirely on the FMA and
// integer pipes (no MUFU, no conversion instruction).  m is an integer and
// c2 = (kShift - m, kShift - m), so t = s scale + c2 = kShift + n with
// n = round(s scale - m) and f = s scale - m - n in [-1/2, 1/2]; 2^f is a
// cubic (coefficients fitted here for minimum relative error, 7.5e-5), and
// its fp32 bit pattern becomes fp16 bits by rounding off 13 mantissa bits and
// rebasing the exponent, with n added to the exponent field (t's low bits
// hold n).  Results below 2^-14 (fp16 subnormals) flush to 0 or less than
// 2^-14; masked scores carry a finite sentinel whose n is hugely negative.
__device__ __forceinline__ uint32_t exp2_pair_fma(float a, float b, uint64_t scale2, uint64_t c2) {
  const uint64_t sv = pk2(a, b);
  const uint64_t t = f32x2_fma(sv, scale2, c2);
  const uint64_t d = f32x2_add(c2, t ^ 0x8000000080000000ull);  // -(m + n)
  const uint64_t f = f32x2_fma(sv, scale2, d);
  uint64_t p = f32x2_fma(f, pk2(0.05517132207751274f), pk2(0.24261054396629333f));
  p = f32x2_fma(p, f, pk2(0.6932609677314758f));
  p = f32x2_fma(p, f, pk2(0.9999281167984009f));
  // fp16 bits: ((p + 2^12 - 0x38000000) >> 13) + (n << 10), clamped at 0
  const int h0 = max((int)(((uint32_t)p - 0x37FFF000u) >> 13) + (int)((uint32_t)t << 10), 0);
  const int h1 = max((int)(((uint32_t)(p >> 32) - 0x37FFF000u) >> 13) + (int)((uint32_t)(t >> 32) << 10), 0);
  return __byte_perm((uint32_t)h0, (uint32_t)h1, 0x5410);
}

// all lanes of the warp wait; false on every lane if any lane's wait ran out
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, tc05::mbar_wait(bar, parity));
}

}  // namespace attn_tc

__device__ int g_attn_tc05_error;

// POLY8: of every 8 exponent pairs, this many run on the FMA and integer
// pipes (exp2_pair_fma), the rest as paired fp16 ex2 on the MUFU pipe
template <int POLY8>
__global__ void __launch_bounds__(attn_tc::NTHREADS, 2)
attn_tc05_kernel(const __half* __restrict__ q, const __half* __restrict__ kc, const __half* __restrict__ vc, int H,
                 int Tq, int ctx, int start_pos, float scale_log2, __half* __restrict__ o) {
  using namespace attn_tc;
  using namespace tc05;
  constexpr int HD = 16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int half = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kend = start_pos + Tq;
  const int nqt = (Tq + 127) >> 7;
  int tiles[4];
  const int ntile = cta_tiles(half, nqt, tiles);
  if (ntile == 0) return;  // uniform over the CTA
  int nkb = 0;             // 64-key blocks this CTA's tiles see
  for (int i = 0; i < ntile; ++i) nkb = max(nkb, tile_blocks(tiles[i], start_pos, kend));
  const int nkb_all = (kend + 63) >> 6;  // layout of the launch (shared-memory size)

  unsigned char* Qs = smem + OFF_Q;
  unsigned char* Ones = smem + OFF_ONES;
  unsigned char* Ks = smem + OFF_K;
  unsigned char* Vt = smem + vt_offset(nkb_all);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bar_offset(nkb_all));
  // per softmax warpgroup w: S written (MMA commit), S read (its 128 threads),
  // P written (its 128 threads), P V complete (MMA commit)
  uint64_t* s_full = bars;
  uint64_t* s_free = bars + 2;
  uint64_t* p_full = bars + 4;
  uint64_t* pv_done = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }

  // ---- stage K, Q, V^T and the ones tile ----
  const size_t bh = (size_t)b * H + h;
  const __half* kb = kc + bh * ctx * HD;
  const __half* vb = vc + bh * ctx * HD;
  const __half* qb = q + bh * Tq * HD;
  const uint32_t sQ = smem_u32(Qs), sK = smem_u32(Ks), sV = smem_u32(Vt), sOnes = smem_u32(Ones);
  for (int i = threadIdx.x; i < nkb * 64 * 2; i += NTHREADS) {
    const int key = i >> 1, c = i & 1;
    const int r = key & 63, slot = (key >> 6) & 3, sb = key >> 8;
    const bool in = key < kend;
    cp_async16(Ks + sb * KSUPER_BYTES + sw_off(r, 2 * slot + c), kb + (size_t)(in ? key : 0) * HD + c * 8,
               in ? 16 : 0);
  }
  for (int i = threadIdx.x; i < ntile * 128 * 2; i += NTHREADS) {
    const int slot = i >> 8, r = (i >> 1) & 127, c = i & 1;
    const int row = tiles[slot] * 128 + r;
    const bool in = row < Tq;
    cp_async16(Qs + sw_off(r, 2 * slot + c), qb + (size_t)(in ? row : 0) * HD + c * 8, in ? 16 : 0);
  }
  cp_async_commit();
  // V^T: item = (block, 8-key chunk, dim pair): 8 rows of two dims -> two 16-byte
  // chunks; all loads of a thread are issued before its stores
  {
    constexpr int VITEMS = (MAX_KEYS + NTHREADS - 1) / NTHREADS;
    uint32_t w[VITEMS][8];
#pragma unroll
    for (int it = 0; it < VITEMS; ++it) {
      const int i = threadIdx.x + it * NTHREADS;
      const int dp = i & 7, key0 = (i >> 3) * 8;  // (block, chunk) = i >> 3
#pragma unroll
      for (int e = 0; e < 8; ++e)
        w[it][e] = (i < nkb * 64 && key0 + e < kend)
                       ? __ldg(reinterpret_cast<const uint32_t*>(vb + (size_t)(key0 + e) * HD) + dp)
                       : 0u;
    }
#pragma unroll
    for (int it = 0; it < VITEMS; ++it) {
      const int i = threadIdx.x + it * NTHREADS;
      if (i < nkb * 64) {
        const int dp = i & 7, ch = (i >> 3) & 7, blk = i >> 6;
        const uint32_t base = sV + blk * VT_BLOCK_BYTES;
        st_shared_v4(base + sw_off(2 * dp, ch), __byte_perm(w[it][0], w[it][1], 0x5410),
                     __byte_perm(w[it][2], w[it][3], 0x5410), __byte_perm(w[it][4], w[it][5], 0x5410),
                     __byte_perm(w[it][6], w[it][7], 0x5410));
        st_shared_v4(base + sw_off(2 * dp + 1, ch), __byte_perm(w[it][0], w[it][1], 0x7632),
                     __byte_perm(w[it][2], w[it][3], 0x7632), __byte_perm(w[it][4], w[it][5], 0x7632),
                     __byte_perm(w[it][6], w[it][7], 0x7632));
      }
    }
  }
  for (int i = threadIdx.x; i < ONES_BYTES / 16; i += NTHREADS)
    st_shared_v4(sOnes + i * 16, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
  cp_async_wait<0>();
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  ATTN_TC_TRACE(7, 0);
  const uint32_t tmem = *tmem_slot;

  if (warp == MMA_WARP) {
    if (lane == 0) {
      // ---- MMA issue for both warpgroups, round r: S of step r + 1 once S of
      // step r has been read, then P V of step r once P of step r is written ----
      constexpr uint32_t IDESC_S = idesc_f16(false, 128, 64);
      constexpr uint32_t IDESC_PV = idesc_f16(false, 128, 16);
      const uint64_t dOnes = sw128_desc(sOnes);
      int nsl[2] = {0, 0}, sl[2][4], tot[2] = {0, 0};
      for (int i = 0; i < ntile; ++i) {
        const int w = tile_owner(i, ntile);
        sl[w][nsl[w]++] = i;
        tot[w] += tile_blocks(tiles[i], start_pos, kend);
      }
      int sk[2] = {0, 0}, sj[2] = {0, 0};  // next S: tile (index into sl) and key block
      int pk[2] = {0, 0}, pj[2] = {0, 0};  // next P V
      auto issue_s = [&](int w) {
        const int slot = sl[w][sk[w]];
        const uint64_t da = sw128_desc(sQ) + 2 * slot;
        const uint64_t db = sw128_desc(sK + (sj[w] >> 2) * KSUPER_BYTES) + 2 * (sj[w] & 3);
        umma_f16(tmem + w * WG_COLS + COL_S, da, db, IDESC_S, 0);
        umma_commit(&s_full[w]);
        if (++sj[w] == tile_blocks(tiles[slot], start_pos, kend)) {
          sj[w] = 0;
          ++sk[w];
        }
      };
      auto issue_pv = [&](int w) {
        const int slot = sl[w][pk[w]];
        const uint64_t dV = sw128_desc(sV + pj[w] * VT_BLOCK_BYTES);
        const uint32_t tw = tmem + w * WG_COLS;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (pj[w] | kk) != 0;
          umma_f16_ts(tw + COL_O, tw + COL_P + 8 * kk, dV + 2 * kk, IDESC_PV, acc);
          umma_f16_ts(tw + COL_SUM, tw + COL_P + 8 * kk, dOnes + 2 * kk, IDESC_PV, acc);
        }
        umma_commit(&pv_done[w]);
        if (++pj[w] == tile_blocks(tiles[slot], start_pos, kend)) {
          pj[w] = 0;
          ++pk[w];
        }
      };
      for (int w = 0; w < 2; ++w)
        if (tot[w] > 0) issue_s(w);
      const int rounds = max(tot[0], tot[1]);
      bool ok = true;
      for (int r = 0; r < rounds && ok; ++r) {
        for (int w = 0; w < 2 && ok; ++w)
          if (r + 1 < tot[w]) {
            ok = mbar_wait(&s_free[w], (uint32_t)(r & 1));
            fence_after_sync();
            ATTN_TC_TRACE(5, r + 1);
            if (ok) issue_s(w);
          }
        for (int w = 0; w < 2 && ok; ++w)
          if (r < tot[w]) {
            ok = mbar_wait(&p_full[w], (uint32_t)(r & 1));
            fence_after_sync();
            ATTN_TC_TRACE(6, r);
            if (ok) issue_pv(w);
          }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---- softmax: warpgroup wg, thread = query row 32 (warp % 4) + lane of its
    // current tile (tensor-memory lane quarter warp % 4) ----
    const int wg = warp >> 2, qw = warp & 3;
    const uint32_t tb = tmem + wg * WG_COLS + ((uint32_t)(qw * 32) << 16);
    const int rr = qw * 32 + lane;
    int g = 0;  // steps of this warpgroup
    bool ok = true;
    for (int i = 0; i < ntile && ok; ++i) {
      if (tile_owner(i, ntile) != wg) continue;
      const int t = tiles[i];
      const int nb = tile_blocks(t, start_pos, kend);
      const int qpos = start_pos + t * 128 + rr;
      float m = 0.f;  // reference maximum, exp2 domain, an integer
      for (int j = 0; j < nb; ++j, ++g) {
        if (!warp_wait(&s_full[wg], (uint32_t)(g & 1))) {
          ok = false;
          break;
        }
        fence_after_sync();
        ATTN_TC_TRACE(0, g);
        float s[64];
        tmem_ld32_nowait(tb + COL_S, s);
        tmem_ld32_nowait(tb + COL_S + 32, s + 32);
        tmem_wait_ld();
        fence_before_sync();
        mbar_arrive(&s_free[wg]);  // the MMA may overwrite S now
        ATTN_TC_TRACE(1, g);
        const int k0 = j * 64;
        if (k0 + 63 > start_pos + t * 128 || k0 + 64 > kend) {
          const int nvis = min(qpos + 1, kend) - k0;  // keys of this block the row sees
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= nvis) s[c] = kMasked;
        }
        float mx[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int c = 4; c < 64; c += 8) {
          mx[0] = fmax3(mx[0], s[c], s[c + 4]);
          mx[1] = fmax3(mx[1], s[c + 1], s[c + 5]);
          mx[2] = fmax3(mx[2], s[c + 2], s[c + 6]);
          mx[3] = fmax3(mx[3], s[c + 3], s[c + 7]);
        }
        const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
        bool pv_waited = g == 0;
        if (j == 0) {
          // first step of the tile: key 0 is visible to every row; O and the row
          // sum restart (the P V MMAs of this step overwrite them).  m is kept
          // an integer: P <= 2^(1/2) at the maximum, rescale factors are exact.
          m = rintf(mt);
        } else {
          const bool mv = mt > m + 8.f;
          if (__any_sync(0xffffffffu, mv)) {
            // O and the row sum must hold step g - 1 before they are rescaled
            if (!warp_wait(&pv_done[wg], (uint32_t)((g - 1) & 1))) {
              ok = false;
              break;
            }
            pv_waited = true;
            fence_after_sync();
            const float mn = rintf(mt);
            const float c = mv ? ex2_f32(m - mn) : 1.f;
            if (mv) m = mn;
            float acc[16];
            tmem_ld16(tb + COL_O, acc);
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] *= c;
            tmem_st16(tb + COL_O, acc);
            tmem_ld16(tb + COL_SUM, acc);
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] *= c;
            tmem_st16(tb + COL_SUM, acc);
          }
        }
        const uint64_t scale2 = pk2(scale_log2), c2 = pk2(kShift - m);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t pf[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int cc = 16 * hh + c;
            if ((cc & 7) < POLY8) {
              pf[c] = exp2_pair_fma(s[2 * cc], s[2 * cc + 1], scale2, c2);
            } else {
              const float2 x = ffma2(s[2 * cc], s[2 * cc + 1], scale_log2, -m);
              pf[c] = ex2_f16x2(pack_f16(x.x, x.y));
            }
          }
          if (hh == 0) {
            ATTN_TC_TRACE(2, g);
            // P is free once P V of step g - 1 has completed
            if (!pv_waited && !warp_wait(&pv_done[wg], (uint32_t)((g - 1) & 1))) {
              ok = false;
              break;
            }
            fence_after_sync();
            ATTN_TC_TRACE(3, g);
          }
          tmem_st16u(tb + COL_P + 16 * hh, pf);
        }
        if (!ok) break;
        tmem_wait_st();
        fence_before_sync();
        mbar_arrive(&p_full[wg]);
        ATTN_TC_TRACE(4, g);
      }
      if (!ok) break;
      // tile done: O / row sum -> o[b, row, h, :]
      if (!warp_wait(&pv_done[wg], (uint32_t)((g - 1) & 1))) {
        ok = false;
        break;
      }
      fence_after_sync();
      float ov[16], sm[16];
      tmem_ld16(tb + COL_O, ov);
      tmem_ld16(tb + COL_SUM, sm);
      const int row = t * 128 + rr;
      if (row < Tq) {
        const float inv = 1.0f / sm[0];
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) pk[e] = pack_f16_sat(ov[2 * e] * inv, ov[2 * e + 1] * inv);
        uint4* dst = reinterpret_cast<uint4*>(o + (((size_t)b * Tq + row) * H + h) * HD);
        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      fence_before_sync();
    }
    if (!ok) *abort_flag = 1;
  }
  __syncwarp();
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_attn_tc05_error, (int)WALSH_ERR_TIMEOUT);
  if (warp == MMA_WARP) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// Hybrid prefill attention (fp16, head dim 16): S = Q K^T of a 128-row query
// block and 64 keys per step as one tcgen05 MMA into tensor memory; the
// softmax and O += P V stay in registers on mma.sync.  The 16x256b form of
// tcgen05.ld hands a warp its 16 rows of S in exactly the m16n8 accumulator
// layout (thread t: rows t/4 and t/4 + 8, columns 2 (t % 4) .. of each
// 8-column group), so the softmax code is that of attn_head_kernel.  Taking
// S off the mma.sync pipe leaves it 12 of the 20 legacy MMAs per 1024 scores
// (P V and the row sums).
// CTA = one (batch, head); its Q (scaled into the exp2 domain) and K are
// staged packed four 64-row blocks to a 128-byte swizzled row (as in
// attn_tc05_kernel), V as 32-byte rows with the two 16-byte halves swapped
// on every other group of four rows (conflict-free ldmatrix.trans).  Warp 8
// allocates tensor memory and issues the S MMAs into NBUF rotating 64-column
// S buffers; warp w < 8 owns tensor memory lanes 32 (w % 4) + 16 (w / 4) ..
// + 15 of each block (its lane quarter, which is also its scheduler
// partition) and skips the key steps its rows cannot see.  SWAP: odd query
// blocks are staged with their two 64-row halves exchanged, so the diagonal
// step only the lower half sees alternates between partitions 0-1 and 2-3.
// ---------------------------------------------------------------------------
namespace attn_hy {
constexpr int NSOFT = 8, MMA_WARP = 8, NTHREADS = 32 * (NSOFT + 1);
constexpr int MAX_KEYS = 1024, MAX_QB = 8;
constexpr int QSUPER_BYTES = 128 * 128;  // 4 query blocks of 128 rows
constexpr int KSUPER_BYTES = 64 * 128;   // 4 key blocks of 64 rows
__host__ __device__ inline int q_bytes(int nqb) { return (nqb + 3) / 4 * QSUPER_BYTES; }
__host__ __device__ inline int k_off(int nqb) { return q_bytes(nqb); }
__host__ __device__ inline int v_off(int nqb, int nkb) { return k_off(nqb) + (nkb + 3) / 4 * KSUPER_BYTES; }
__host__ __device__ inline int bar_off(int nqb, int nkb) { return v_off(nqb, nkb) + nkb * 64 * 32; }
__host__ inline int smem_bytes(int nqb, int nkb) { return 1024 + bar_off(nqb, nkb) + 128; }  // barriers, tmem slot, abort flag
// byte offset of 16-byte chunk c (0, 1) of V row r
__device__ __forceinline__ uint32_t v_swz(int r, int c) { return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4)); }
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, float (*s)[4]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) s[i][k] = __uint_as_float(r[4 * i + k]);
}
__device__ __forceinline__ int block_steps(int qb, int start_pos, int kend) {
  return (min(kend, start_pos + 128 * qb + 128) + 63) >> 6;
}
}  // namespace attn_hy

template <int NBUF, bool SWAP>
__global__ void __launch_bounds__(attn_hy::NTHREADS, 2)
attn_hybrid_kernel(const __half* __restrict__ q, const __half* __restrict__ kc, const __half* __restrict__ vc, int H,
                   int Tq, int ctx, int start_pos, float scale_log2, __half* __restrict__ o) {
  using namespace attn_hy;
  using namespace tc05;
  constexpr int HD = 16, KT = 64;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int h = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int kend = start_pos + Tq;
  const int nqb = (Tq + 127) >> 7, nkb = (kend + 63) >> 6;
  unsigned char* Qs = smem;
  unsigned char* Ks = smem + k_off(nqb);
  unsigned char* Vs = smem + v_off(nqb, nkb);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bar_off(nqb, nkb));
  constexpr uint32_t TMEM_COLS = 64 * NBUF;
  uint64_t* s_full = bars;         // [NBUF] S buffer written (MMA commit)
  uint64_t* s_free = bars + NBUF;  // [NBUF] S buffer read by the 8 softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (threadIdx.x == 0) {
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], NSOFT);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  // ---- stage K (packed), V (swizzled rows, zero past kend) and Q (scaled, packed) ----
  const size_t bh = (size_t)b * H + h;
  const __half* kb = kc + bh * ctx * HD;
  const __half* vb = vc + bh * ctx * HD;
  const __half* qb = q + bh * Tq * HD;
  for (int i = threadIdx.x; i < nkb * 64 * 2; i += NTHREADS) {
    const int key = i >> 1, c = i & 1;
    const int r = key & 63, slot = (key >> 6) & 3, sb = key >> 8;
    const bool in = key < kend;
    cp_async16(Ks + sb * KSUPER_BYTES + attn_tc::sw_off(r, 2 * slot + c), kb + (size_t)(in ? key : 0) * HD + c * 8,
               in ? 16 : 0);
    cp_async16(Vs + v_swz(key, c), vb + (size_t)(in ? key : 0) * HD + c * 8, in ? 16 : 0);
  }
  cp_async_commit();
  {
    const __half2 sc = __float2half2_rn(scale_log2);
    for (int i = threadIdx.x; i < nqb * 128 * 2; i += NTHREADS) {
      const int qbk = i >> 8, r = (i >> 1) & 127, c = i & 1;
      const int row = qbk * 128 + (SWAP ? (r + 64 * (qbk & 1)) & 127 : r);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < Tq) {
        v = __ldg(reinterpret_cast<const uint4*>(qb + (size_t)row * HD + c * 8));
        __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) hv[e] = __hmul2(hv[e], sc);
      }
      *reinterpret_cast<uint4*>(Qs + (qbk >> 2) * QSUPER_BYTES + attn_tc::sw_off(r, 2 * (qbk & 3) + c)) = v;
    }
  }
  cp_async_wait<0>();
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_f16(false, 128, 64);
      const uint32_t sQ = smem_u32(Qs), sK = smem_u32(Ks);
      int g2 = 0;
      bool ok = true;
      for (int qbk = 0; qbk < nqb && ok; ++qbk) {
        const int nst = block_steps(qbk, start_pos, kend);
        for (int j = 0; j < nst; ++j, ++g2) {
          const int sb = g2 % NBUF;
          if (g2 >= NBUF && !mbar_wait_sleep(&s_free[sb], (uint32_t)((g2 / NBUF - 1) & 1))) {
            ok = false;
            break;
          }
          fence_after_sync();
          const uint64_t da = sw128_desc(sQ + (qbk >> 2) * QSUPER_BYTES) + 2 * (qbk & 3);
          const uint64_t db = sw128_desc(sK + (j >> 2) * KSUPER_BYTES) + 2 * (j & 3);
          umma_f16(tmem + 64 * sb, da, db, IDESC, 0);
          umma_commit(&s_full[sb]);
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    const int r0 = 32 * (warp & 3) + 16 * (warp >> 2);  // this warp's 16 rows of each block
    const uint32_t tl = tmem + ((uint32_t)r0 << 16);
    int g2 = 0;
    bool ok = true;
    for (int qbk = 0; qbk < nqb && ok; ++qbk) {
      const int nst = block_steps(qbk, start_pos, kend);
      const int q0 = qbk * 128 + (SWAP ? (r0 + 64 * (qbk & 1)) & 127 : r0);
      const int r_lo = q0 + g, r_hi = r_lo + 8;
      const int qp_lo = start_pos + r_lo, qp_hi = start_pos + r_hi;
      const int nkey = min(kend, start_pos + q0 + 16);  // keys visible to some row of the slab
      float m_lo = 0.f, m_hi = 0.f;
      float thr_lo = -CUDART_INF_F, thr_hi = -CUDART_INF_F;
      float oacc[HD / 8 + 1][4];
#pragma unroll
      for (int jj = 0; jj < HD / 8 + 1; ++jj) oacc[jj][0] = oacc[jj][1] = oacc[jj][2] = oacc[jj][3] = 0.f;
      for (int j = 0; j < nst; ++j, ++g2) {
        const int sb = g2 % NBUF;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (uint32_t)((g2 / NBUF) & 1)))) {
          ok = false;
          break;
        }
        fence_after_sync();
        float s[KT / 8][4];
        tmem_ld_16x256b_x8(tl + 64 * sb, s);
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        const int k0 = j * KT;
        if (k0 >= nkey) continue;  // no row of this slab sees these keys
        if (k0 + KT > start_pos + q0 || k0 + KT > kend) {
#pragma unroll
          for (int n = 0; n < KT / 8; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = k0 + n * 8 + 2 * t4 + e;
              if (key > qp_lo || key >= kend) s[n][e] = -CUDART_INF_F;
              if (key > qp_hi || key >= kend) s[n][2 + e] = -CUDART_INF_F;
            }
        }
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
        // the reference maximum m of a row moves to the row maximum once it passes
        // m + thr (thr = -inf before the row's first visible key, 8 after)
        const bool mv_lo = mt_lo > m_lo + thr_lo, mv_hi = mt_hi > m_hi + thr_hi;
        if (__any_sync(0xffffffffu, mv_lo || mv_hi)) {
          const float c_lo = !mv_lo ? 1.f : (thr_lo == -CUDART_INF_F ? 0.f : ex2_f32(m_lo - mt_lo));
          const float c_hi = !mv_hi ? 1.f : (thr_hi == -CUDART_INF_F ? 0.f : ex2_f32(m_hi - mt_hi));
#pragma unroll
          for (int jj = 0; jj < HD / 8 + 1; ++jj) {
            oacc[jj][0] *= c_lo; oacc[jj][1] *= c_lo;
            oacc[jj][2] *= c_hi; oacc[jj][3] *= c_hi;
          }
          if (mv_lo) { m_lo = mt_lo; thr_lo = 8.f; }
          if (mv_hi) { m_hi = mt_hi; thr_hi = 8.f; }
        }
        uint32_t pf[KT / 16][4];
        const uint64_t one2 = f2_dup(1.f), nm_lo = f2_dup(-m_lo), nm_hi = f2_dup(-m_hi);
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
          const uint64_t d_lo = f2_fma(f2_pack(s[n][0], s[n][1]), one2, nm_lo);
          const uint64_t d_hi = f2_fma(f2_pack(s[n][2], s[n][3]), one2, nm_hi);
          pf[n >> 1][(n & 1) * 2 + 0] =
              ex2_f16x2(pack_f16(__uint_as_float((uint32_t)d_lo), __uint_as_float((uint32_t)(d_lo >> 32))));
          pf[n >> 1][(n & 1) * 2 + 1] =
              ex2_f16x2(pack_f16(__uint_as_float((uint32_t)d_hi), __uint_as_float((uint32_t)(d_hi >> 32))));
        }
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          uint32_t vf[4];
          ldsm_x4_t(vf, Vs + v_swz(k0 + kk * 16 + (lane & 15), lane >> 4));
          mma_f16(oacc[0], pf[kk], vf[0], vf[1]);
          mma_f16(oacc[1], pf[kk], vf[2], vf[3]);
          mma_f16(oacc[HD / 8], pf[kk], 0x3C003C00u, 0x3C003C00u);  // row sums of P
        }
      }
      if (!ok) break;
      const float inv_lo = 1.0f / oacc[HD / 8][0], inv_hi = 1.0f / oacc[HD / 8][2];
#pragma unroll
      for (int jj = 0; jj < HD / 8; ++jj) {
        const int d = jj * 8 + 2 * t4;
        if (r_lo < Tq)
          *reinterpret_cast<uint32_t*>(o + (((size_t)b * Tq + r_lo) * H + h) * HD + d) =
              pack_f16_sat(oacc[jj][0] * inv_lo, oacc[jj][1] * inv_lo);
        if (r_hi < Tq)
          *reinterpret_cast<uint32_t*>(o + (((size_t)b * Tq + r_hi) * H + h) * HD + d) =
              pack_f16_sat(oacc[jj][2] * inv_hi, oacc[jj][3] * inv_hi);
      }
    }
    if (!ok) *abort_flag = 1;
  }
  __syncwarp();
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_attn_tc05_error, (int)WALSH_ERR_TIMEOUT);
  if (warp == MMA_WARP) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Off by default: measured on B200 (B64 x H32 x T1024, hd 16) the tcgen05
// kernel takes 556-580 us and the hybrid 455 us against 381 us for the
// mma.sync whole-head kernel.  At head dim 16 the work is the 1.2 G softmax
// exponentials per layer: ex2 runs at 16 results / clock / SM whether paired
// (f16x2) or not, a floor of about 260 us; none of the kernels fills that
// pipe (about 50 % busy, latency stalls first), and the whole-head kernel
// issues the fewest instructions per score and holds the most warps per SM.
static int g_attn_tc05 = 0;
static int g_attn_poly8 = -1;  // exponent pairs of 8 on the FMA pipe (WALSH_ATTN_TC_POLY8, default 0)

// 1 when the tcgen05 kernel ran, 0 when it does not apply, negative on error.
int launch_attn_tc05(const void* q, const void* kc, const void* vc, int B, int H, int Tq, int ctx, int start_pos,
                     float scale_log2, void* o, cudaStream_t s) {
  using namespace attn_tc;
  const int kend = start_pos + Tq;
  if (!g_attn_tc05 || Tq <= 4 || Tq > MAX_QTILES * 128 || kend > MAX_KEYS || H > 65535 || B > 65535) return 0;
  if (((((uintptr_t)q) | ((uintptr_t)kc) | ((uintptr_t)vc) | ((uintptr_t)o)) & 15u) != 0) return 0;
  if (g_attn_tc05 == 2) {
    // two or four S buffers, halves exchanged or not: 454-457 us at B64 x H32 x T1024
    const int hs = attn_hy::smem_bytes((Tq + 127) / 128, (kend + 63) / 64);
    auto* kern = attn_hybrid_kernel<2, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, hs) != cudaSuccess)
      return launch_status();
    kern<<<dim3(H, B), attn_hy::NTHREADS, hs, s>>>((const __half*)q, (const __half*)kc, (const __half*)vc, H, Tq, ctx,
                                                   start_pos, scale_log2, (__half*)o);
    const int e = launch_status();
    return e == WALSH_OK ? 1 : e;
  }
  const int smem = smem_bytes((kend + 63) / 64);
  if (g_attn_poly8 < 0) {
    const char* e = getenv("WALSH_ATTN_TC_POLY8");
    g_attn_poly8 = e ? atoi(e) : 0;
    g_attn_poly8 = g_attn_poly8 < 0 ? 0 : (g_attn_poly8 > 6 ? 6 : g_attn_poly8);
  }
  auto kern = attn_tc05_kernel<0>;
  switch (g_attn_poly8) {
    case 1: kern = attn_tc05_kernel<1>; break;
    case 2: kern = attn_tc05_kernel<2>; break;
    case 3: kern = attn_tc05_kernel<3>; break;
    case 4: kern = attn_tc05_kernel<4>; break;
    case 5: kern = attn_tc05_kernel<5>; break;
    case 6: kern = attn_tc05_kernel<6>; break;
    default: break;
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status();
  kern<<<dim3(2, H, B), NTHREADS, smem, s>>>((const __half*)q, (const __half*)kc, (const __half*)vc, H, Tq, ctx,
                                             start_pos, scale_log2, (__half*)o);
  const int e = launch_status();
  return e == WALSH_OK ? 1 : e;
}

int attn_tc05_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_tc05_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_attn_tc05_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace walsh

extern "C" int walsh_attn_set_path(int tcgen05) {
  const int prev = walsh::g_attn_tc05;
  walsh::g_attn_tc05 = tcgen05 == 2 ? 2 : (tcgen05 ? 1 : 0);
  return prev;
}
