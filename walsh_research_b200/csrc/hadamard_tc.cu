// Hadamard-32 algebra on the tensor cores (bf16 activations in HBM, 32 x 16
// layout, i.e. C = 512 with in_o = out_o = 16).
//
// Per token the HadamardLinear map (src/model/fht_cuda.py:489-519) is
//   Z = H Xa (32x32 +-1 contraction over the groups), V_g = W_g Z_g (32
//   independent 16x16 ternary mat-vecs), Y = H V,  y = beta . Y / 32,
// and the Hadamard head mixer (src/model/fht_cuda.py:652-670) is the same
// chain with dense per-head W and beta shared by the heads.  Each warp owns
// 16 tokens whose rows sit in shared memory as bf16 [32][16] blocks:
//   stage 1/3  per token: A = block^T via ldmatrix.trans, B = H (registers),
//              4 n-tiles x 2 k-steps of m16n8k16, result stored back
//              transposed with stmatrix.trans (block <- H-mixed block);
//   stage 2    per group g: A = the 16 tokens' g-th 16-wide slice, B = W_g^T
//              (fp16 copy [g][o][i], read through L1), result stored back.
// The MMA operands are fp16 (H and the ternary weights are exact in fp16;
// intermediates keep 11 significant bits), accumulation is fp32, and the
// 1/32 normalisation is applied after the first transform so the staged
// values stay far inside the fp16 range (conversions saturate at +-65504).
#include "common.cuh"
#include "mma.cuh"

namespace walsh {

constexpr int kTcC = 512;
constexpr int kTcRow = kTcC + 8;  // padded smem row of one token (bf16 elements)
constexpr int kTcTok = 16;        // tokens per warp

struct TcQkvEpilogue {
  int T, n_head, hd, ctx, start_pos;
  const float* cos;
  const float* sin;
};

// B fragments of H (symmetric, +-1) for K = 32 (2 k-steps) x N = 32 (4 n-tiles).
__device__ __forceinline__ void hadamard_bfrags(uint32_t (&hb)[2][4][2]) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int n = 8 * nt + gid;
        const int k0 = 16 * ks + 8 * half + 2 * t4;
        const uint32_t lo = (__popc(k0 & n) & 1) ? 0xBC00u : 0x3C00u;  // fp16 -1 / +1
        const uint32_t hi = (__popc((k0 + 1) & n) & 1) ? 0xBC00u : 0x3C00u;
        hb[ks][nt][half] = lo | (hi << 16);
      }
}

// rowp[32][16] (fp16) <- k * H-mixed rowp: C[i][g] = sum_g' rowp[g'][i] H[g'][g], stored as rowp[g][i].
__device__ __forceinline__ void fht_tc_token(__half* rowp, const uint32_t (&hb)[2][4][2], float k) {
  const int lane = threadIdx.x & 31;
  uint32_t a[2][4];
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
    ldsm_x4_t(a[ks], rowp + (16 * ks + (lane & 7) + ((lane >> 4) << 3)) * 16 + ((lane >> 3) & 1) * 8);
  float c[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) mma_f16(c[nt], a[ks], hb[ks][nt][0], hb[ks][nt][1]);
  }
  __syncwarp();
  const int m = lane >> 3, j = lane & 7;
#pragma unroll
  for (int np = 0; np < 2; ++np) {
    const int nt = 2 * np;
    stsm_x4_t(rowp + (8 * (nt + (m >> 1)) + j) * 16 + (m & 1) * 8, pack_f16_sat(k * c[nt][0], k * c[nt][1]),
              pack_f16_sat(k * c[nt][2], k * c[nt][3]), pack_f16_sat(k * c[nt + 1][0], k * c[nt + 1][1]),
              pack_f16_sat(k * c[nt + 1][2], k * c[nt + 1][3]));
  }
  __syncwarp();
}

// tile[t][g*16 + o] <- sum_i W[g][o][i] tile[t][g*16 + i] for the warp's 16 tokens (fp16).
__device__ __forceinline__ void group_mma(__half* tile, const __half* __restrict__ wt) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, t4 = lane & 3;
  const int m = lane >> 3, j = lane & 7;
#pragma unroll 4
  for (int g = 0; g < 32; ++g) {
    uint32_t a[4];
    ldsm_x4(a, tile + (lane & 15) * kTcRow + g * 16 + (lane >> 4) * 8);
    float c[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const __half* wr = wt + ((size_t)g * 16 + 8 * nt + gid) * 16 + 2 * t4;
      c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
      mma_f16(c[nt], a, __ldg(reinterpret_cast<const unsigned int*>(wr)),
              __ldg(reinterpret_cast<const unsigned int*>(wr + 8)));
    }
    __syncwarp();
    stsm_x4(tile + (j + (m & 1) * 8) * kTcRow + g * 16 + (m >> 1) * 8, pack_f16_sat(c[0][0], c[0][1]),
            pack_f16_sat(c[0][2], c[0][3]), pack_f16_sat(c[1][0], c[1][1]), pack_f16_sat(c[1][2], c[1][3]));
  }
  __syncwarp();
}

// Full Hadamard chain on the warp's tile: H (then * 1/32), grouped W, H.
__device__ __forceinline__ void hadamard_chain(__half* tile, const __half* __restrict__ wt,
                                               const uint32_t (&hb)[2][4][2]) {
#pragma unroll 1
  for (int t = 0; t < kTcTok; ++t) fht_tc_token(tile + t * kTcRow, hb, 1.0f / 32.0f);
  group_mma(tile, wt);
#pragma unroll 1
  for (int t = 0; t < kTcTok; ++t) fht_tc_token(tile + t * kTcRow, hb, 1.0f);
}

// Stage 16 bf16 token rows of src (row stride kTcC) into the tile (row stride kTcRow, still bf16
// bits), zero-filling past ntok.
template <typename TIN>
__device__ __forceinline__ void stage_rows(__half* dst, const TIN* __restrict__ src, int64_t tok0, int64_t ntok) {
  const int lane = threadIdx.x & 31;
#pragma unroll 4
  for (int i = lane; i < kTcTok * (kTcC / 8); i += 32) {
    const int r = i / (kTcC / 8), c = i - r * (kTcC / 8);
    const bool in = tok0 + r < ntok;
    cp_async16(dst + r * kTcRow + c * 8, src + (in ? (tok0 + r) * kTcC : 0) + c * 8, in ? 16 : 0);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncwarp();
}

// In place: TIN (bf16 or fp16) bits -> fp16(x * s[c]) (s may be NULL -> 1).
template <typename TIN>
__device__ __forceinline__ void scale_rows_to_f16(__half* tile, const float* __restrict__ s) {
  const int lane = threadIdx.x & 31;
  for (int i = lane; i < kTcTok * (kTcC / 2); i += 32) {
    const int r = i >> 8, c = (i & 255) * 2;
    uint32_t* p = reinterpret_cast<uint32_t*>(tile + r * kTcRow + c);
    const float2 v = unpack2<TIN>(*p);
    const float s0 = s ? __ldg(s + c) : 1.f, s1 = s ? __ldg(s + c + 1) : 1.f;
    *p = pack_f16_sat(v.x * s0, v.y * s1);
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------
// HadamardLinear (plain): y = out_scale * beta . H W H (alpha . x) / 32
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128)
hlin_tc_kernel(const __nv_bfloat16* __restrict__ x, int64_t ntok, const __half* __restrict__ wt,
               const float* __restrict__ alpha, const float* __restrict__ beta, float out_scale,
               __nv_bfloat16* __restrict__ y) {
  extern __shared__ float4 smem4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __half* tile = reinterpret_cast<__half*>(smem4) + warp * kTcTok * kTcRow;
  const int64_t tok0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * kTcTok;
  uint32_t hb[2][4][2];
  hadamard_bfrags(hb);
  stage_rows(tile, x, tok0, ntok);
  scale_rows_to_f16<__nv_bfloat16>(tile, alpha);
  hadamard_chain(tile, wt, hb);
  for (int t = 0; t < kTcTok; ++t) {
    const int64_t tok = tok0 + t;
    if (tok >= ntok) break;
    for (int cp = lane; cp < kTcC / 2; cp += 32) {
      const int c = 2 * cp;
      const float2 v = unpack_f16(*reinterpret_cast<const uint32_t*>(tile + t * kTcRow + c));
      *reinterpret_cast<uint32_t*>(y + tok * kTcC + c) =
          pack_bf16(v.x * __ldg(beta + c) * out_scale, v.y * __ldg(beta + c + 1) * out_scale);
    }
  }
}

// ---------------------------------------------------------------------------
// q/k/v + RoPE + KV-cache write; weights fp16 [32][16][16], alpha/beta [512].
// ---------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(128)
qkv_tc_kernel(const __half* __restrict__ u, int64_t ntok, const __half* __restrict__ wq,
              const __half* __restrict__ wk, const __half* __restrict__ wv, const float* __restrict__ aq,
              const float* __restrict__ ak, const float* __restrict__ av, const float* __restrict__ bq,
              const float* __restrict__ bk, const float* __restrict__ bv, __half* __restrict__ q,
              __half* __restrict__ kc, __half* __restrict__ vc, TcQkvEpilogue ep) {
  constexpr int HALF = HD / 2;
  static_assert(HD % 8 == 0 && 256 % HD == 0, "a lane's 8 channels lie in one head");
  extern __shared__ float4 smem4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __half* tile = reinterpret_cast<__half*>(smem4) + warp * kTcTok * kTcRow;
  const int64_t tok0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * kTcTok;
  uint32_t hb[2][4][2];
  hadamard_bfrags(hb);
  // gridDim.y == 3: one projection per CTA (small token counts); else all three
  const int set_lo = gridDim.y == 3 ? (int)blockIdx.y : 0, set_hi = gridDim.y == 3 ? set_lo + 1 : 3;
#pragma unroll 1
  for (int set = set_lo; set < set_hi; ++set) {
    const float* al = set == 0 ? aq : (set == 1 ? ak : av);
    const float* be = set == 0 ? bq : (set == 1 ? bk : bv);
    const __half* wt = set == 0 ? wq : (set == 1 ? wk : wv);
    __half* dst = set == 0 ? q : (set == 1 ? kc : vc);
    stage_rows(tile, u, tok0, ntok);  // re-read per projection (L2-resident); keeps one tile per warp
    scale_rows_to_f16<__half>(tile, al);
    hadamard_chain(tile, wt, hb);
    // epilogue: lane owns channels c = 256 * pass + 8 * lane .. +7 (one head, dims d0..d0+7)
    float bl[2][8];
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const float4 lo = __ldg(reinterpret_cast<const float4*>(be + pass * 256 + lane * 8));
      const float4 hi = __ldg(reinterpret_cast<const float4*>(be + pass * 256 + lane * 8 + 4));
      bl[pass][0] = lo.x; bl[pass][1] = lo.y; bl[pass][2] = lo.z; bl[pass][3] = lo.w;
      bl[pass][4] = hi.x; bl[pass][5] = hi.y; bl[pass][6] = hi.z; bl[pass][7] = hi.w;
    }
    const int d0 = (lane * 8) % HD;
    for (int t = 0; t < kTcTok; ++t) {
      const int64_t tok = tok0 + t;
      if (tok >= ntok) break;
      const int b = (int)(tok / ep.T), tt = (int)(tok - (int64_t)b * ep.T);
      float cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
      if (set < 2) {
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(ep.cos + (size_t)tt * HALF + (d0 >> 1)));
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(ep.sin + (size_t)tt * HALF + (d0 >> 1)));
        cs[0] = c4.x; cs[1] = c4.y; cs[2] = c4.z; cs[3] = c4.w;
        sn[0] = s4.x; sn[1] = s4.y; sn[2] = s4.z; sn[3] = s4.w;
      }
      const size_t plane = set == 0 ? (size_t)ep.T : (size_t)ep.ctx;  // rows per head plane
      const size_t row = set == 0 ? (size_t)tt : (size_t)(ep.start_pos + tt);
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int c = pass * 256 + lane * 8;
        const int head = c / HD;
        const uint4 v = *reinterpret_cast<const uint4*>(tile + t * kTcRow + c);
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
        uint32_t ow[4];
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          const float2 f = unpack_f16(vw[q2]);
          const float v0 = f.x * bl[pass][2 * q2], v1 = f.y * bl[pass][2 * q2 + 1];
          ow[q2] = pack_f16_sat(v0 * cs[q2] - v1 * sn[q2], v0 * sn[q2] + v1 * cs[q2]);
        }
        *reinterpret_cast<uint4*>(dst + (((size_t)b * ep.n_head + head) * plane + row) * HD + d0) =
            make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Attention output: head mixer (optional) + wo + mHC site epilogue.
//   o [ntok][512] token-major attention output (32 heads x 16)
//   mixer: Y = beta_m[d] . H (W_h) H o / 32; then wo: f = beta_o . H W_o H (alpha_o . Y) / 32
//   x_out[i] = sum_j H_res[i][j] x[j] + H_post[i] f   (x, x_out [ntok][4][512]; may alias)
// ---------------------------------------------------------------------------
template <typename TX>
__global__ void __launch_bounds__(128)
attn_out_tc_kernel(const __half* __restrict__ o, int64_t ntok, const __half* __restrict__ wmix,
                   const float* __restrict__ beta_mix, const __half* __restrict__ wo,
                   const float* __restrict__ alpha_o, const float* __restrict__ beta_o, const TX* x,
                   const float* __restrict__ hmix, TX* xo) {
  extern __shared__ float4 smem4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __half* tile = reinterpret_cast<__half*>(smem4) + warp * kTcTok * kTcRow;
  const int64_t tok0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * kTcTok;
  uint32_t hb[2][4][2];
  hadamard_bfrags(hb);
  stage_rows(tile, o, tok0, ntok);
  if (wmix) {
    hadamard_chain(tile, wmix, hb);
    // head-mixer output scale beta_m[d] fused with wo's input scale alpha_o[c]
    for (int i = lane; i < kTcTok * (kTcC / 2); i += 32) {
      const int r = i >> 8, c = (i & 255) * 2;
      uint32_t* p = reinterpret_cast<uint32_t*>(tile + r * kTcRow + c);
      const float2 v = unpack_f16(*p);
      *p = pack_f16_sat(v.x * __ldg(beta_mix + (c & 15)) * __ldg(alpha_o + c),
                        v.y * __ldg(beta_mix + ((c + 1) & 15)) * __ldg(alpha_o + c + 1));
    }
    __syncwarp();
  } else {
    scale_rows_to_f16<__half>(tile, alpha_o);
  }
  hadamard_chain(tile, wo, hb);
  // epilogue: lane owns channels c = 256 * pass + 8 * lane .. +7; 16-byte loads and stores
  float bo[2][8];
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const float4 lo = __ldg(reinterpret_cast<const float4*>(beta_o + pass * 256 + lane * 8));
    const float4 hi = __ldg(reinterpret_cast<const float4*>(beta_o + pass * 256 + lane * 8 + 4));
    bo[pass][0] = lo.x; bo[pass][1] = lo.y; bo[pass][2] = lo.z; bo[pass][3] = lo.w;
    bo[pass][4] = hi.x; bo[pass][5] = hi.y; bo[pass][6] = hi.z; bo[pass][7] = hi.w;
  }
  // software-pipelined over the warp's 16 tokens: token t + 1's stream rows and
  // mixing coefficients are loaded before token t is computed and stored (the
  // tokens' rows are disjoint, so this is safe when xo aliases x)
  uint4 xq[2][4];
  float4 hq[5];  // H_post[4] | H_res[16]
  auto load_tok = [&](int64_t tok, uint4 (&xr)[2][4], float4 (&hr4)[5]) {
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const size_t base = (size_t)tok * 4 * kTcC + pass * 256 + lane * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j) xr[pass][j] = *reinterpret_cast<const uint4*>(x + base + (size_t)j * kTcC);
    }
    const float4* h4 = reinterpret_cast<const float4*>(hmix + tok * kMapRows + 4);
#pragma unroll
    for (int i = 0; i < 5; ++i) hr4[i] = __ldg(h4 + i);
  };
  if (tok0 < ntok) load_tok(tok0, xq, hq);
  for (int t = 0; t < kTcTok; ++t) {
    const int64_t tok = tok0 + t;
    if (tok >= ntok) break;
    uint4 xn[2][4];
    float4 hn[5];
    if (t + 1 < kTcTok && tok + 1 < ntok) load_tok(tok + 1, xn, hn);
    const float hp[4] = {hq[0].x, hq[0].y, hq[0].z, hq[0].w};
    const float hr[16] = {hq[1].x, hq[1].y, hq[1].z, hq[1].w, hq[2].x, hq[2].y, hq[2].z, hq[2].w,
                          hq[3].x, hq[3].y, hq[3].z, hq[3].w, hq[4].x, hq[4].y, hq[4].z, hq[4].w};
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const int c = pass * 256 + lane * 8;
      const size_t base = (size_t)tok * 4 * kTcC + c;
      const uint4 v = *reinterpret_cast<const uint4*>(tile + t * kTcRow + c);
      const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
      uint32_t ow[4][4];
#pragma unroll
      for (int q2 = 0; q2 < 4; ++q2) {
        const float2 f = unpack_f16(vw[q2]);
        const float f0 = f.x * bo[pass][2 * q2], f1 = f.y * bo[pass][2 * q2 + 1];
        float2 xf[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xf[j] = unpack2<TX>((&xq[pass][j].x)[q2]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float* r = hr + 4 * i;
          const float a0 = (((r[0] * xf[0].x + r[1] * xf[1].x) + r[2] * xf[2].x) + r[3] * xf[3].x) + hp[i] * f0;
          const float a1 = (((r[0] * xf[0].y + r[1] * xf[1].y) + r[2] * xf[2].y) + r[3] * xf[3].y) + hp[i] * f1;
          ow[i][q2] = pack2<TX>(a0, a1);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(xo + base + (size_t)i * kTcC) = make_uint4(ow[i][0], ow[i][1], ow[i][2], ow[i][3]);
    }
#pragma unroll
    for (int pass = 0; pass < 2; ++pass)
#pragma unroll
      for (int j = 0; j < 4; ++j) xq[pass][j] = xn[pass][j];
#pragma unroll
    for (int i = 0; i < 5; ++i) hq[i] = hn[i];
  }
}

static inline int smem_set(const void* fn, int bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess ? 0 : -1;
}

static inline bool al16(const void* p) { return (((uintptr_t)p) & 15u) == 0; }

}  // namespace walsh

using namespace walsh;

// Warps (16 tokens each) per CTA: 4 normally; 1 when the token count would
// leave most SMs idle (decode steps).
static int tc_warps_per_cta(int64_t ntok) { return ntok >= 148 * 4 * kTcTok ? 4 : 1; }

extern "C" walsh_status walsh_hadamard_linear_tc_fwd(const void* x, int64_t ntok, const void* w_f16,
                                                     float w_scale, const float* alpha, const float* beta, void* y,
                                                     void* stream) {
  if (int e = injected("hadamard_linear_tc_fwd")) return e;
  WALSH_CHECK_ARG(x && w_f16 && alpha && beta && y);
  WALSH_CHECK_SHAPE(ntok >= 0);
  WALSH_CHECK_ARG(al16(x) && al16(y) && al16(w_f16));
  if (ntok == 0) return WALSH_OK;
  const int smem = 4 * kTcTok * kTcRow * (int)sizeof(__half);
  if (smem_set((const void*)hlin_tc_kernel, smem)) return WALSH_ERR_LAUNCH;
  const unsigned grid = (unsigned)((ntok + 63) / 64);
  hlin_tc_kernel<<<grid, 128, smem, (cudaStream_t)stream>>>((const __nv_bfloat16*)x, ntok, (const __half*)w_f16,
                                                            alpha, beta, w_scale, (__nv_bfloat16*)y);
  return launch_status();
}

extern "C" walsh_status walsh_attn_qkv_tc_fwd(const void* u, int B, int T, int n_head, const void* wq_f16,
                                              const float* wq_alpha, const float* wq_beta, const void* wk_f16,
                                              const float* wk_alpha, const float* wk_beta, const void* wv_f16,
                                              const float* wv_alpha, const float* wv_beta, const float* rope_cos,
                                              const float* rope_sin, int n_pos, int start_pos, void* q,
                                              void* k_cache, void* v_cache, int ctx, void* stream) {
  if (int e = injected("attn_qkv_tc_fwd")) return e;
  WALSH_CHECK_ARG(u && wq_f16 && wq_alpha && wq_beta && wk_f16 && wk_alpha && wk_beta && wv_f16 && wv_alpha &&
                  wv_beta && rope_cos && rope_sin && q && k_cache && v_cache);
  WALSH_CHECK_SHAPE(B > 0 && T > 0 && n_head > 0 && kTcC % n_head == 0);
  const int hd = kTcC / n_head;
  WALSH_CHECK_SHAPE((hd == 16 || hd == 32) && start_pos >= 0 && start_pos + T <= ctx && T <= n_pos);
  WALSH_CHECK_ARG(al16(u) && al16(wq_f16) && al16(wk_f16) && al16(wv_f16));
  WALSH_CHECK_ARG(al16(q) && al16(k_cache) && al16(v_cache) && al16(wq_beta) && al16(wk_beta) && al16(wv_beta) &&
                  al16(rope_cos) && al16(rope_sin));
  const int64_t ntok = (int64_t)B * T;
  const int wpc = tc_warps_per_cta(ntok);
  const int smem = 4 * kTcTok * kTcRow * (int)sizeof(__half);
  TcQkvEpilogue ep{T, n_head, hd, ctx, start_pos, rope_cos, rope_sin};
  const dim3 grid((unsigned)((ntok + wpc * kTcTok - 1) / (wpc * kTcTok)), wpc == 4 ? 1 : 3);
  auto kern = hd == 16 ? qkv_tc_kernel<16> : qkv_tc_kernel<32>;
  if (smem_set((const void*)kern, smem)) return WALSH_ERR_LAUNCH;
  kern<<<grid, 32 * wpc, wpc * kTcTok * kTcRow * sizeof(__half), (cudaStream_t)stream>>>(
      (const __half*)u, ntok, (const __half*)wq_f16, (const __half*)wk_f16, (const __half*)wv_f16, wq_alpha,
      wk_alpha, wv_alpha, wq_beta, wk_beta, wv_beta, (__half*)q, (__half*)k_cache, (__half*)v_cache, ep);
  return launch_status();
}

extern "C" walsh_status walsh_attn_out_tc_fwd(const void* o, int64_t ntok, const void* wmix_f16,
                                              const float* beta_mix, const void* wo_f16, const float* wo_alpha,
                                              const float* wo_beta, const void* x, int x_dtype, const float* hmix,
                                              void* x_out, void* stream) {
  if (int e = injected("attn_out_tc_fwd")) return e;
  WALSH_CHECK_ARG(o && wo_f16 && wo_alpha && wo_beta && x && hmix && x_out);
  WALSH_CHECK_ARG(!wmix_f16 || beta_mix);
  WALSH_CHECK_SHAPE(ntok >= 0);
  WALSH_CHECK_DTYPE(x_dtype);
  WALSH_CHECK_SHAPE(x_dtype == WALSH_BF16 || x_dtype == WALSH_F16);
  WALSH_CHECK_ARG(al16(o) && al16(wo_f16) && (!wmix_f16 || al16(wmix_f16)) && al16(x) && al16(x_out) &&
                  al16(wo_beta) && al16(hmix));
  if (ntok == 0) return WALSH_OK;
  const int wpc = tc_warps_per_cta(ntok);
  const int smem = 4 * kTcTok * kTcRow * (int)sizeof(__half);
  const unsigned grid = (unsigned)((ntok + wpc * kTcTok - 1) / (wpc * kTcTok));
  const size_t dsmem = wpc * kTcTok * kTcRow * sizeof(__half);
  cudaStream_t s = (cudaStream_t)stream;
  if (x_dtype == WALSH_F16) {
    if (smem_set((const void*)attn_out_tc_kernel<__half>, smem)) return WALSH_ERR_LAUNCH;
    attn_out_tc_kernel<__half><<<grid, 32 * wpc, dsmem, s>>>((const __half*)o, ntok, (const __half*)wmix_f16,
                                                            beta_mix, (const __half*)wo_f16, wo_alpha, wo_beta,
                                                            (const __half*)x, hmix, (__half*)x_out);
  } else {
    if (smem_set((const void*)attn_out_tc_kernel<__nv_bfloat16>, smem)) return WALSH_ERR_LAUNCH;
    attn_out_tc_kernel<__nv_bfloat16><<<grid, 32 * wpc, dsmem, s>>>(
        (const __half*)o, ntok, (const __half*)wmix_f16, beta_mix, (const __half*)wo_f16, wo_alpha, wo_beta,
        (const __nv_bfloat16*)x, hmix, (__nv_bfloat16*)x_out);
  }
  return launch_status();
}
