/*
 * libwalsh — C ABI of the B200 (sm_100a) kernels for Walsh's forward hot path.
 *
 * The reference (pulseofthemachine/Walsh-Research) has no FFI: its "plugin"
 * boundary is Python module substitution inside src/model (the import-time
 * choice at src/model/physics.py:84-91, the factories at
 * src/model/chassis.py:54-94).  Each entry point below replaces the forward
 * of one reference module or one fused group of them; the reference
 * interface it stands in for is cited beside it.  The Python package
 * walsh_research_b200.model re-exposes them behind the reference's class
 * names and state-dict keys.
 *
 * Conventions
 *  - All pointers are device pointers unless stated otherwise; every buffer
 *    is allocated and owned by the caller.  Nothing here allocates device
 *    memory on the forward path, frees caller memory or synchronises.
 *  - Activations are float32 (dtype WALSH_F32), bfloat16 (WALSH_BF16) or
 *    float16 (WALSH_F16); arithmetic is float32 (tensor-core kernels: fp16 or
 *    bf16 operands, fp32 accumulation).  The model's bfloat16 mode keeps the
 *    residual stream in bf16 and the normalised activations it feeds the
 *    layers (u, q/k/v, attention output) in fp16.
 *  - Every call launches on `stream` (a cudaStream_t passed as void*) and
 *    returns a walsh_status: 0 on success, a negative code on a rejected
 *    argument (checked on the host before any launch) or a launch failure.
 *  - Ternary weights are 2 bits each in the reference's encoding
 *    (-1 -> 00, 0 -> 01, +1 -> 10; four per byte, first value in the most
 *    significant bits; src/model/fht_cuda.py:65-93), rows of length K padded
 *    to ceil(K/4) bytes with the zero code.
 */
#ifndef WALSH_H_
#define WALSH_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int walsh_status;

enum {
  WALSH_OK = 0,
  WALSH_ERR_ARG = -1,      /* null pointer / bad scalar argument */
  WALSH_ERR_SHAPE = -2,    /* unsupported or inconsistent sizes */
  WALSH_ERR_DTYPE = -3,    /* unknown dtype code */
  WALSH_ERR_ALIGN = -4,    /* pointer not aligned as required */
  WALSH_ERR_LAUNCH = -5,   /* CUDA launch error */
  WALSH_ERR_TIMEOUT = -6,  /* a bounded device-side wait gave up */
  WALSH_ERR_INJECTED = -7, /* host-side fault injector fired (tests) */
  WALSH_ERR_NOT_INIT = -8, /* library not initialised for this device */
  WALSH_ERR_INDEX = -9,    /* a device kernel saw an out-of-range token id */
  WALSH_ERR_SCRATCH = -10  /* problem larger than an allocation-free entry point's fixed scratch */
};

enum { WALSH_F32 = 0, WALSH_BF16 = 1, WALSH_F16 = 2 };

/* Human-readable text of a status code (static storage). */
const char* walsh_status_str(walsh_status s);
/* ABI version of this library (bumped on any signature change). */
int walsh_abi_version(void);

/* ---------------------------------------------------------------------------
 * Ternary weights (load-time)
 * ------------------------------------------------------------------------- */

/* Absmean ternary quantisation + 2-bit packing of a latent weight tensor
 * viewed as [rows, k]: gamma = mean|W| + 1e-8 over the whole tensor,
 * q = clamp(round_half_even(W / gamma), -1, 1).  Writes packed
 * [rows, ceil(k/4)] and gamma (one device float).
 * Replaces physics.quantize_ternary (src/model/physics.py:13-51) and
 * moe.quantize_ternary (src/model/moe.py:268-303; the scaled form is
 * q * gamma, i.e. the same q with gamma applied by the consumer) followed by
 * pack_ternary_weights (src/model/fht_cuda.py:65-93). */
walsh_status walsh_ternary_quantize_pack(const float* w, int64_t rows, int k,
                                         uint8_t* packed, float* gamma, void* stream);

/* Unpack [rows, ceil(k/4)] -> float [rows, k].
 * Replaces unpack_ternary_weights (src/model/fht_cuda.py:96-117). */
walsh_status walsh_ternary_unpack(const uint8_t* packed, int64_t rows, int k, float* out,
                                  void* stream);

/* ---------------------------------------------------------------------------
 * Hadamard-32 algebra
 * ------------------------------------------------------------------------- */

/* y[t] = w_scale * beta . H . W_q . H . (alpha . x[t]) for ntok tokens, with x
 * viewed as [32 groups, in_o] and y as [32, out_o]; H is the Sylvester
 * Hadamard matrix / sqrt(32).  w2bit: [32, out_o, ceil(in_o/4)], alpha:
 * [32, in_o], beta: [32, out_o] (float32).  Supported (in_o, out_o):
 * 16x16, 64x64, 16x64, 64x16.
 * Replaces HadamardLinear.forward (src/model/fht_cuda.py:489-519) and
 * HadamardTernaryLinearTuple.forward (src/model/fht_cuda.py:550-569). */
walsh_status walsh_hadamard_linear_fwd(const void* x, int x_dtype, int64_t ntok, int in_o,
                                       int out_o, const uint8_t* w2bit, float w_scale,
                                       const float* alpha, const float* beta, void* y,
                                       int y_dtype, void* stream);

/* Hadamard head mixing on token-major [ntok, n_head, hd]: each group of 32
 * consecutive heads is mixed as y = beta . H (W_h x_h) H with one shared
 * W [32, hd, hd] and beta [hd] (float32).  In-place is allowed.
 * Replaces HadamardHeadMixerFused.forward (src/model/fht_cuda.py:652-670) as
 * called per head group by CausalSelfAttention (src/model/chassis.py:468-477). */
walsh_status walsh_head_mixer_fwd(const void* x, int dtype, int64_t ntok, int n_head, int hd,
                                  const float* W, const float* beta, void* y, void* stream);

/* Fused q/k/v projection + RoPE + KV-cache write for one attention layer.
 * u: [B, T, C] (C = 32*in_o); w*_2bit/alpha/beta as walsh_hadamard_linear_fwd
 * with in_o = out_o = C/32; rope_cos/sin: float [n_pos >= T, hd/2], row t
 * rotating token t (the real and imaginary parts of the reference's
 * freqs_cis buffer, offset by the caller to the first token's position).
 * Writes q: [B, H, T, hd] and k, v into the caches [B, H, ctx, hd] at
 * positions start_pos..start_pos+T-1, all in out_dtype (u is in dtype).
 * Replaces CausalSelfAttention.forward lines 426-440 (src/model/chassis.py):
 * wq/wk/wv, apply_rotary_emb (src/model/chassis.py:339-345) and
 * KVCache.update (src/model/chassis.py:297-322). */
walsh_status walsh_attn_qkv_fwd(const void* u, int dtype, int B, int T, int C, int n_head,
                                const uint8_t* wq_2bit, const float* wq_alpha, const float* wq_beta,
                                const uint8_t* wk_2bit, const float* wk_alpha, const float* wk_beta,
                                const uint8_t* wv_2bit, const float* wv_alpha, const float* wv_beta,
                                const float* rope_cos, const float* rope_sin, int n_pos,
                                int start_pos, void* q, void* k_cache, void* v_cache, int ctx,
                                int out_dtype, void* stream);

/* Causal attention over the KV cache: query t (position start_pos+t) sees
 * keys 0..start_pos+t, scale 1/sqrt(hd).  q: [B, H, T, hd]; caches
 * [B, H, ctx, hd]; o: token-major [B, T, H, hd].  hd in {16, 32}.
 * Replaces the scaled_dot_product_attention calls of
 * CausalSelfAttention.forward (src/model/chassis.py:442-466). */
walsh_status walsh_attn_fwd(const void* q, const void* k_cache, const void* v_cache, int dtype,
                            int B, int H, int T, int hd, int ctx, int start_pos, void* o,
                            void* stream);

/* Tensor-core forms for bfloat16 activations with C = 512 (32 groups x 16):
 * each 32-point transform is a +-1 32x32 MMA contraction, the per-group
 * ternary mat-vecs are grouped MMAs (fp16 operands, fp32 accumulation).
 * Weights are fp16 copies laid out [32 groups][out 16][in 16] (ternary values
 * for HadamardLinear; for the head mixer the transpose of W[h][i][o]).  All
 * pointers 16-byte aligned.
 *
 * walsh_hadamard_linear_tc_fwd: y = w_scale * beta . H W H (alpha . x), x and
 * y bfloat16 [ntok, 512].  Replaces HadamardLinear.forward
 * (src/model/fht_cuda.py:489-519). */
walsh_status walsh_hadamard_linear_tc_fwd(const void* x, int64_t ntok, const void* w_f16,
                                          float w_scale, const float* alpha, const float* beta,
                                          void* y, void* stream);

/* walsh_attn_qkv_tc_fwd: walsh_attn_qkv_fwd for C = 512 on the tensor cores
 * (same layouts and RoPE/cache semantics; weights as above); u, q and the
 * caches are fp16. */
walsh_status walsh_attn_qkv_tc_fwd(const void* u, int B, int T, int n_head, const void* wq_f16,
                                   const float* wq_alpha, const float* wq_beta, const void* wk_f16,
                                   const float* wk_alpha, const float* wk_beta, const void* wv_f16,
                                   const float* wv_alpha, const float* wv_beta,
                                   const float* rope_cos, const float* rope_sin, int n_pos,
                                   int start_pos, void* q, void* k_cache, void* v_cache, int ctx,
                                   void* stream);

/* walsh_attn_out_tc_fwd: for the fp16 attention output o [ntok, 512]
 * (token-major, 32 heads x 16) and a 16-bit residual stream x (x_dtype
 * WALSH_BF16 or WALSH_F16): optional Hadamard head mixing (wmix_f16 = W^T per head,
 * beta_mix [16]; NULL skips it), the wo HadamardLinear, and the mHC site
 * epilogue x_out = H_res x + H_post f (x, x_out [ntok, 4, 512], may alias;
 * hmix as walsh_mhc_map).  Replaces CausalSelfAttention.forward lines
 * 468-483 (src/model/chassis.py) and mHCResidualStream.forward lines 366-381
 * (src/model/mhc.py). */
walsh_status walsh_attn_out_tc_fwd(const void* o, int64_t ntok, const void* wmix_f16,
                                   const float* beta_mix, const void* wo_f16,
                                   const float* wo_alpha, const float* wo_beta, const void* x,
                                   int x_dtype, const float* hmix, void* x_out, void* stream);

/* ---------------------------------------------------------------------------
 * mHC residual streams (n_streams = 4)
 * ------------------------------------------------------------------------- */

/* Site prologue for x: [ntok, 4, C]:
 *   r = rsqrt(mean(x^2) + map_eps) over all 4C values;
 *   d = phi . (r x) with phi [24, 4C] = rows of H_pre | H_post | H_res;
 *   H_pre = sigmoid(a0 d[0:4] + b[0:4]), H_post = 2 sigmoid(a1 d[4:8] + b[4:8]),
 *   H_res = Sinkhorn_20(a2 d[8:24] + b[8:24]) (exp, then column and row
 *   normalisation with eps 1e-8);
 *   u = sum_j H_pre[j] x_j, then (if norm_w != NULL) the chassis RMSNorm
 *   u / sqrt(mean(u^2) + norm_eps) * norm_w.
 * mparams: float [28] = {a_pre, a_post, a_res, unused, b_pre[4], b_post[4],
 * b_res[16]}.  phi_lp (optional, may be NULL): a copy of phi in x's 16-bit
 * type (bfloat16 for bf16 x, float16 for fp16 x); with it, a 16-bit x selects
 * the tensor-core kernel (C = 512 or 2048).  phi_frag (optional): phi_lp
 * rearranged into mma.sync B-fragment order, [4C/16 k-steps][32 lanes][3
 * n-tiles][2 regs] of packed 16-bit pairs (element (n, k) with n = 8 nt + lane/4,
 * k = 16 ks + 8 reg + 2 (lane%4) + {0,1}); with it, C = 512 and 16-bit x/u select
 * the single-pass kernel that reads x once (TMA).  u is written in u_dtype (the
 * model's 16-bit mode writes fp16).  Writes u [ntok, C] and hmix float [ntok, 24] =
 * {H_pre[4], H_post[4], H_res[16] row-major}.
 * Replaces ResidualStreamMapping.forward x3 and the pre-mix of
 * mHCResidualStream.forward (src/model/mhc.py:283-318, 345-364) plus the
 * attention_norm / ffn_norm RMSNorm of mHCLlamaBlock (src/model/mhc.py:514-523). */
walsh_status walsh_mhc_map(const void* x, int dtype, int64_t ntok, int C, const float* phi,
                           const void* phi_lp, const void* phi_frag, const float* mparams,
                           float map_eps, const float* norm_w, float norm_eps, void* u, int u_dtype,
                           float* hmix, void* stream);

/* Status word of the single-pass map kernels' bounded TMA waits (0 or
 * WALSH_ERR_TIMEOUT); synchronous read, reset != 0 clears it.  No counterpart
 * in the reference. */
int walsh_map_error(int reset);

/* Kernel choice of walsh_mhc_map for C = 512, 16-bit x and at least 9472
 * tokens when phi_frag is given: on != 0 the persistent pipelined
 * single-pass kernel (x read from HBM once; the default), 0 the two-pass
 * tensor-core kernel (x read twice).  on < 0 only queries.  Returns the
 * previous setting.  Process-wide; for comparisons.  No counterpart in the
 * reference. */
int walsh_map_set_pipe(int on);

/* Site epilogue: x_out[i] = sum_j H_res[i][j] x[j] + H_post[i] f for each
 * token (x, x_out: [ntok, 4, C]; f: [ntok, C]; x_out may alias x).
 * Replaces mHCResidualStream.forward lines 366-381 (src/model/mhc.py). */
walsh_status walsh_mhc_post(const void* x, const void* f, const float* hmix, int dtype,
                            int64_t ntok, int C, void* x_out, void* stream);

/* Sinkhorn-Knopp projection of n 4x4 matrices (float32), exp then `iters`
 * (column, row) normalisations with `eps`.
 * Replaces SinkhornKnopp.forward (src/model/mhc.py:214-229). */
walsh_status walsh_sinkhorn(const float* h, int64_t n, int iters, float eps, float* out,
                            void* stream);

/* ---------------------------------------------------------------------------
 * Hadamard MoE
 * ------------------------------------------------------------------------- */

/* Router + experts for u: [ntok, C], E = C/32 experts of hidden 128:
 *   p = softmax(W2 silu(W1 u)) with w1t = W1 transposed, [C, C/4], and
 *   w2 = W2 [E, C/4] (float32);
 *   top_k largest p selected (ties to the lower index), weights w = p/sum;
 *   y[e] = w_e * gd * Dq silu(gg Gq u_e) * (gu Uq u_e) for selected e, 0 else,
 *   where u_e is the e-th 32-wide block and Gq/Uq [E,128,32], Dq [E,32,128]
 *   are 2-bit ternary with gammas {gg, gu, gd} (device float[3]).
 * Router-only call: gate/up/down/gammas all NULL (only the optional mask,
 * probs and weights outputs are written).
 * When weights_in (float [ntok, E]) is not NULL the router is skipped (w1t,
 * w2 may be NULL) and
 * every expert with a non-zero weight in it is evaluated with that weight
 * (FastMoEExperts with caller-given routing weights; mask/probs/weights
 * outputs are then not written).
 * When fuse_post != 0, `y` is not written; instead the mHC site epilogue is
 * applied: x_out = H_res x + H_post y (x, x_out [ntok, 4, C] in x_dtype, hmix
 * as walsh_mhc_map; x_out may alias x).  mask_out (uint8 [ntok, E]), probs_out
 * and weights_out (float [ntok, E]) are optional (NULL to skip).
 * tc (host pointer, may be NULL): bf16/fp16 copies of the weights; with bf16
 * or fp16 u, C = 512 and a bf16 stream they select the tensor-core kernel (router and
 * experts on m16n8k16 MMAs; all experts evaluated densely and weighted by
 * the routing weight, zero outside the top-k, as the reference does).
 * Replaces HadamardRouter.forward (src/model/moe.py:418-447),
 * FastMoEExperts.forward (src/model/moe.py:337-380) and HadamardMoE.forward
 * (src/model/moe.py:512-542) followed by the ffn-site epilogue of
 * mHCResidualStream.forward (src/model/mhc.py:366-381). */
/* Expert selection of the MoE entry points below (pass NULL for the
 * reference's rule).
 * WALSH_ROUTE_TOPK: top_k experts by router probability, ties to the lower
 *   expert index -- what HadamardRouter.forward runs (src/model/moe.py:432-436).
 * WALSH_ROUTE_THRESHOLD: every expert whose probability exceeds `threshold`,
 *   at least `min_experts` and at most top_k of them, taken in descending
 *   probability -- the rule HadamardRouter's docstring and constructor
 *   arguments describe (threshold, min_experts, max_experts;
 *   src/model/moe.py:383-403) but its forward does not apply.  Opt-in.
 * In both modes the routing weights are renormalised over the selected
 * experts.  WALSH_ERR_ARG for an unknown mode, min_experts outside
 * [1, top_k] or a threshold outside [0, 1]. */
enum { WALSH_ROUTE_TOPK = 0, WALSH_ROUTE_THRESHOLD = 1 };
typedef struct {
  int mode;
  int min_experts;
  float threshold;
} walsh_moe_routing;

typedef struct {   /* all in the dtype of u (bf16 or fp16) */
  const void* w1;   /* [C/4, C]   router layer 1 (nn.Linear layout) */
  const void* w2;   /* [E, C/4]   router layer 2 */
  const void* gate; /* [E, 128, 32] ternary values, gamma not applied */
  const void* up;   /* [E, 128, 32] */
  const void* down; /* [E, 32, 128] */
} walsh_moe_tc_weights;

walsh_status walsh_moe_fwd(const void* u, int dtype, int64_t ntok, int C, int top_k,
                           const float* w1t, const float* w2, const uint8_t* gate_2bit,
                           const uint8_t* up_2bit, const uint8_t* down_2bit, const float* gammas,
                           void* y, int fuse_post, const void* x, int x_dtype, const float* hmix,
                           void* x_out, const float* weights_in, uint8_t* mask_out,
                           float* probs_out, float* weights_out, const walsh_moe_tc_weights* tc,
                           const walsh_moe_routing* routing, void* stream);

/* MoE after router layer 1 (for decode-sized token counts): hpre = u W1^T
 * [ntok, C/4] (u's dtype, computed by the caller, e.g. walsh_octo_linear_fwd
 * with the router's W1 and unit scales); then per token silu, logits =
 * W2 silu(hpre), softmax, top_k experts (ties to the lower index), weights
 * renormalised over the selected experts, only the selected ternary experts,
 * and either y (fuse_post = 0) or the mHC site epilogue into x_out (as for
 * walsh_moe_fwd).  C = 512 or 2048; w2 float32 [E, C/4] 16-byte aligned;
 * expert weights as for walsh_moe_fwd.  mask/probs/weights optional.
 * Replaces HadamardRouter.forward layer 2 onward and HadamardMoE.forward
 * (src/model/moe.py:418-447, 337-380, 512-542). */
walsh_status walsh_moe_hidden_fwd(const void* u, const void* hpre, int dtype, int64_t ntok, int C,
                                  int top_k, const float* w2, const uint8_t* gate_2bit,
                                  const uint8_t* up_2bit, const uint8_t* down_2bit,
                                  const float* gammas, void* y, int fuse_post, const void* x,
                                  int x_dtype, const float* hmix, void* x_out, uint8_t* mask_out,
                                  float* probs_out, float* weights_out, const walsh_moe_routing* routing,
                                  void* stream);

/* Prefill-sized MoE for C = 512 (E = 16, router hidden 128) on the
 * 5th-generation tensor cores, in two calls.
 *
 * walsh_moe_router_tc_fwd: h = u W1^T as a tcgen05 GEMM whose epilogue does
 * the rest of the router per token: silu(h) rounded to u's dtype, logits =
 * silu(h) W2^T, softmax, top_k (ties to the lower index), routing weights
 * renormalised over the selected experts.  u [ntok, 512] bf16/fp16; w1
 * [128, 512] and w2 [16, 128] in u's dtype; mask uint8, probs and weights
 * float32 [ntok, 16].  All pointers 16-byte aligned.  Replaces
 * HadamardRouter.forward (src/model/moe.py:418-447). */
walsh_status walsh_moe_router_tc_fwd(const void* u, int dtype, int64_t ntok, const void* w1,
                                     const void* w2, int top_k, uint8_t* mask, float* probs,
                                     float* weights, const walsh_moe_routing* routing, void* stream);

/* walsh_moe_experts_tc_fwd: the 16 ternary SwiGLU experts (all evaluated,
 * weighted by `weights`, 0 outside the top-k) and either y [ntok, 512]
 * (fuse_post = 0, u's dtype) or the mHC site epilogue into x_out (as for
 * walsh_moe_fwd; x bf16/fp16).  w_gu [8, 256, 64]: for expert pair p, rows
 * 0..127 are gate hidden units and 128..255 up hidden units, columns 0..31
 * expert 2p's inputs and 32..63 expert 2p + 1's (ternary values in u's
 * dtype); w_down [16, 32, 128]; gammas float[3] (gate, up, down).  All
 * pointers 16-byte aligned.  Replaces FastMoEExperts.forward and the
 * weighted combination of HadamardMoE.forward (src/model/moe.py:337-380,
 * 512-542). */
walsh_status walsh_moe_experts_tc_fwd(const void* u, int dtype, int64_t ntok, const float* weights,
                                      const void* w_gu, const void* w_down, const float* gammas,
                                      void* y, int fuse_post, const void* x, int x_dtype,
                                      const float* hmix, void* x_out, void* stream);

/* ---------------------------------------------------------------------------
 * Octonion (Cayley-Dickson) layers as tensor-core GEMMs
 *
 * w_hi [N, K] is the dense signed expansion of an OctonionTernaryLinear's
 * eight ternary blocks: w[(i, o), (j, k)] = SIGN[i][j] Wq[WIDX[i][j]][o][k]
 * (src/model/constants.py:15-52), exact in fp16/bf16.  w_dtype must be
 * WALSH_F16 for fp16 x and WALSH_BF16 for bf16 or float32 x; w_lo (optional,
 * float32 x only) is a bf16 correction w - w_hi for non-ternary matrices
 * (the folded head mixer).  float32 x is split into bf16 hi + lo in the
 * kernel (float32 accuracy).  scale[n] multiplies output column n (beta of
 * the output part).  K a multiple of 8, N even, x/w 16-byte aligned.
 * ------------------------------------------------------------------------- */

/* 16-bit x runs on the 5th-generation tensor cores (TMA-staged operands,
 * tcgen05.mma into Tensor Memory) unless switched off here; float32 x, and
 * any call with w_lo, use the mma.sync mainloop.  Returns the previous
 * setting.  Process-wide; not thread-safe against concurrent launches.
 * No counterpart in the reference (selects between this library's own two
 * mainloops, e.g. to compare them in tests). */
int walsh_octo_set_mainloop(int tcgen05);
/* Few-row GEMMs (a 256-wide tiling that would occupy at most a quarter of the
 * SMs) run with 64-wide CTA tiles when on (the default); on = 0 keeps the
 * 256-wide tiles, on < 0 only queries.  Returns the previous setting.  A
 * switch for comparisons: both tilings give the same sums. */
int walsh_octo_set_narrow(int on);
/* GEMMs with the plain epilogue (walsh_octo_linear_fwd,
 * walsh_hadamard_linear_dense_fwd) on the tcgen05 kernel stage each scaled
 * 32 x 32 output block in shared memory and write it with a TMA store when
 * on (the default; 16-bit outputs, N a multiple of 32); on = 0 keeps each
 * lane's row stores, on < 0 only queries.  Returns the previous setting.  A
 * switch for comparisons: both give the same bits. */
int walsh_octo_set_tma_store(int on);

/* Status word of the tcgen05 kernels (GEMMs and prefill attention) on the
 * current device: 0, or WALSH_ERR_TIMEOUT once a bounded wait inside one of
 * them gave up (the affected tile is not written).  Synchronous read;
 * reset != 0 clears it.  No counterpart in the reference. */
int walsh_tc05_error(int reset);

/* Kernel of fp16 prefill attention with head dim 16 and at most 1024 keys:
 * 1 = on the 5th-generation tensor cores (S and P V as tcgen05 MMAs into
 * Tensor Memory); 2 = hybrid (S as a tcgen05 MMA, softmax and P V on
 * mma.sync); 0 (the default): the mma.sync kernels of walsh_attn_fwd; any
 * other nonzero value means 1.  Returns the previous setting.  Process-wide.
 * No counterpart in the reference (selects between this library's own
 * kernels, e.g. to compare them in tests). */
int walsh_attn_set_path(int tcgen05);

/* Test hook for the bounded waits: one thread waits on an mbarrier that is
 * never arrived at, gives up after budget_cycles SM clocks (at most 4e9) and
 * sets the walsh_tc05_error status word to WALSH_ERR_TIMEOUT.  The context
 * stays usable.  No counterpart in the reference. */
walsh_status walsh_tc05_wait_selftest(long long budget_cycles, void* stream);

/* y = scale . (x w^T), y in x's dtype [M, N].
 * Replaces OctonionTernaryLinearRef.forward / OctonionFusedLinear.forward
 * (src/model/physics.py:66-82, src/model/cayley_dickson_cuda.py:654-668). */
walsh_status walsh_octo_linear_fwd(const void* x, int dtype, int64_t M, int K, const void* w_hi,
                                   const void* w_lo, int w_dtype, int64_t N, const float* scale,
                                   void* y, void* stream);

/* q/k/v in one GEMM: w [3C, C] = wq | wk | wv rows, scale [3C]; RoPE
 * (interleaved pairs, rope_cos/sin [>= T, hd/2] rows of the tokens' own
 * positions) on q and k; q -> [B, H, T, hd], k/v -> caches [B, H, ctx, hd] at
 * rows start_pos..; outputs in u's dtype.
 * Replaces CausalSelfAttention.forward lines 424-447 for the octonion algebra
 * (src/model/chassis.py:424-447, apply_rotary_emb :339-345). */
walsh_status walsh_octo_qkv_fwd(const void* u, int dtype, int B, int T, int C, int n_head,
                                const void* w_hi, const void* w_lo, int w_dtype, const float* scale,
                                const float* rope_cos, const float* rope_sin, int n_pos, int start_pos,
                                void* q, void* k_cache, void* v_cache, int ctx, void* stream);

/* h = silu(g) * v with g, v the gate/up outputs: w [2 hidden, K] holds the
 * gate and up rows interleaved (row 2j = gate unit j, row 2j+1 = up unit j),
 * scale interleaved the same way; h [M, hidden] in u's dtype.
 * Replaces SwiGLUMLP.forward up to down_proj (src/model/chassis.py:497-505). */
walsh_status walsh_octo_swiglu_fwd(const void* u, int dtype, int64_t M, int K, const void* w_hi,
                                   const void* w_lo, int w_dtype, const float* scale, int64_t hidden,
                                   void* h, void* stream);

/* f = scale . (a w^T) [M, C] followed by the mHC site epilogue
 * x_out[m, i] = sum_j H_res[i][j] x[m, j] + H_post[i] f[m] (x, x_out
 * [M, 4, C] float32 or bfloat16, may alias; hmix as for walsh_mhc_post).
 * Used for wo (with the octonion head mixer folded into w) and down_proj.
 * Replaces SwiGLUMLP down_proj / wo followed by mHCResidualStream's output
 * mixing (src/model/chassis.py:476-483, 505-507; src/model/mhc.py:376-381). */
walsh_status walsh_octo_post_fwd(const void* a, int dtype, int64_t M, int K, const void* w_hi,
                                 const void* w_lo, int w_dtype, const float* scale, int C,
                                 const void* x, int x_dtype, const float* hmix, void* x_out,
                                 void* stream);

/* ---------------------------------------------------------------------------
 * Channel modulation (x viewed as [nseg, seg_len, C], segment = seg_len
 * consecutive rows of the flat [rows, C] tensor, as the reference's
 * x.view(B*n, T, C) at src/model/mhc.py:530)
 * ------------------------------------------------------------------------- */

/* Partial segment sums of the RMSNorm'd rows xn = x/sqrt(mean(x^2)+eps)*norm_w
 * (xn = x when norm_w is NULL):
 * partial[s, c, :] = sum of xn over rows [c*chunk, (c+1)*chunk) of segment s,
 * chunk = walsh_chmod_chunk_rows(seg_len); partial: float [nseg, nchunk, C]. */
int walsh_chmod_chunk_rows(int seg_len);
walsh_status walsh_chmod_stats(const void* x, int dtype, int64_t nrows, int C, int seg_len,
                               const float* norm_w, float norm_eps, float* partial, void* stream);

/* bulk = (sum of partials)/seg_len; h = silu(g1 W1q bulk); m = g2 W2q h;
 * scale = 1 + clamp(scale_temp, 0.1, 0.5) tanh(m[:E]); shift = m[E:].
 * W1q [C/4, C], W2q [2E, C/4] 2-bit ternary, gammas device float[2].
 * Replaces HadamardChannelModulation.forward lines 694-710 and
 * _forward_ternary (src/model/moe.py:694-710, 753-762). */
walsh_status walsh_chmod_mlp(const float* partial, int nseg, int seg_len, int C,
                             const uint8_t* w1_2bit, const uint8_t* w2_2bit,
                             const float* gammas, const float* scale_temp, float* scale,
                             float* shift, void* stream);

/* walsh_chmod_mlp with the first layer on the tensor cores, for large
 * segment counts (batched decode has one segment per stream row): the fp32
 * segment means are split into three bf16 rows (hi + mid + lo = the mean to
 * fp32 precision), one GEMM against W1 as dense bf16 [C/4, C] (the ternary
 * values, exact in bf16; g1 is applied after the three fp32 results are
 * added), then layer 2 as in walsh_chmod_mlp.  scratch: a device buffer of
 * walsh_chmod_mlp_tc_scratch_bytes(nseg, C) bytes, 16-byte aligned.
 * C % 64 == 0.  Replaces the same lines of src/model/moe.py as
 * walsh_chmod_mlp. */
int64_t walsh_chmod_mlp_tc_scratch_bytes(int nseg, int C);
walsh_status walsh_chmod_mlp_tc(const float* partial, int nseg, int seg_len, int C, const void* w1_bf16,
                                const uint8_t* w2_2bit, const float* gammas, const float* scale_temp,
                                void* scratch, float* scale, float* shift, void* stream);

/* out = [x +] xn + r (xn * scale_b + 0.1 shift_b - xn) per 32-wide block b,
 * r = residual_scale (0.5 in mHCLlamaBlock),
 * with xn the RMSNorm'd row (xn = x when norm_w is NULL) and (scale, shift)
 * [nseg, E] of the row's segment; the leading x is added when add_input != 0.
 * out may alias x.
 * Replaces the channel-modulation residual of mHCLlamaBlock.forward
 * (src/model/mhc.py:528-532) with the modulation apply of
 * src/model/moe.py:724-751. */
walsh_status walsh_chmod_apply(const void* x, int dtype, int64_t nrows, int C, int seg_len,
                               const float* norm_w, float norm_eps, const float* scale,
                               const float* shift, float residual_scale, int add_input, void* out,
                               void* stream);

/* Channel modulation of single-row segments (seg_len 1: batched decode, one
 * segment per stream row) in one launch: walsh_chmod_stats + walsh_chmod_mlp
 * + walsh_chmod_apply with the same arguments' meaning, C = 512 only, x and
 * out 16-bit (WALSH_BF16 / WALSH_F16, 16-byte aligned, out may alias x),
 * packed W1 16-byte and W2 4-byte aligned.  scale, shift [nrows, C/32] are written as
 * by walsh_chmod_mlp.  Layer sums in float32 with a different order than the
 * three-step form (results agree to float32 rounding).
 * Replaces HadamardChannelModulation.forward on [B*n, 1, C]
 * (src/model/moe.py:681-762) inside mHCLlamaBlock.forward (src/model/mhc.py:528-532). */
walsh_status walsh_chmod_rows_fwd(const void* x, int dtype, int64_t nrows, int C, const float* norm_w,
                                  float norm_eps, const uint8_t* w1_2bit, const uint8_t* w2_2bit,
                                  const float* gammas, const float* scale_temp, float residual_scale, int add_input,
                                  float* scale, float* shift, void* out, void* stream);

/* Allocation-free channel modulation: stats, mlp and apply above in one call,
 * with the scratch (partial sums, scale, shift) in a fixed device array inside
 * the library instead of caller buffers.  No counterpart in the reference (its
 * PyTorch forward allocates freely); it exists for hosts that cannot allocate
 * device memory at call time.  Arguments mean what they mean for
 * walsh_chmod_stats/_mlp/_apply; out may alias x.
 * Limit: round64(nseg*nchunk*C) + 2*round64(nseg*C/32) <= 1,048,576 floats
 * (4 MiB; nchunk = ceil(seg_len / walsh_chmod_chunk_rows), round64 = round up
 * to a multiple of 64), else WALSH_ERR_SCRATCH before any launch.
 * The first call in a CUDA context (per device, with that device current)
 * looks up the array's address (set-up); make it before any stream capture.
 * The address is cached under the context's process-unique id, so a device
 * reset, or another context made current on the device, is looked up again
 * on its first call (also outside capture).  The array is shared: calls that
 * overlap on the device race and must be ordered by the caller.  Nothing in
 * it needs to start at zero. */
walsh_status walsh_chmod_fwd_noalloc(const void* x, int dtype, int64_t nrows, int C, int seg_len,
                                     const float* norm_w, float norm_eps, const uint8_t* w1_2bit,
                                     const uint8_t* w2_2bit, const float* gammas,
                                     const float* scale_temp, float residual_scale, int add_input,
                                     void* out, void* stream);

/* Part of the tensor-core expert kernel of walsh_moe_experts_tc_fwd: only
 * experts first_expert .. first_expert + n_experts - 1 (whole quarters of 4
 * containing them are evaluated), output y [ntok, 512] in u's dtype with
 * only those quarters' columns written.  For expert parallelism, where a
 * rank evaluates the experts it owns over the rows it received.
 * Replaces FastMoEExperts.forward (src/model/moe.py:337-380) for a subset
 * of the experts. */
walsh_status walsh_moe_experts_tc_part_fwd(const void* u, int dtype, int64_t ntok, const float* weights,
                                           const void* w_gu, const void* w_down, const float* gammas,
                                           int first_expert, int n_experts, void* y, void* stream);

/* ---------------------------------------------------------------------------
 * Expert parallelism over NVLink (HadamardMoE, src/model/moe.py:512-542: expert
 * e consumes and produces only feature block e, lines 536-541).
 *
 * world ranks (one per GPU, world <= 8) each hold ntok tokens (the same ntok
 * on every rank); rank j owns experts [j E/world, (j + 1) E/world), E = C/32.
 * Each rank allocates, in memory its peers can write (walsh_ipc_*), recv_u
 * [world * ntok, C] (u's dtype), recv_w float [world * ntok, E], y_full
 * [ntok, C] (u's dtype) and flags uint32 [2 * world] (zeroed once); and, in
 * its own memory, counters uint32 [2 * world] (zeroed once).  The peer_*
 * arguments are host arrays of world device pointers (this rank's own
 * buffer at index `rank`).  `epoch` (non-zero, the same on every rank, new
 * for every exchange) is the value written to the flags.
 *
 * walsh_ep_dispatch: rows of u and of the routing weights (float [ntok, E])
 * to every rank: the columns of rank j's experts into rank j's recv_u rows
 * rank * ntok .. + ntok - 1, the weights (zero outside rank j's experts)
 * into its recv_w; then flags[rank] = epoch on rank j.
 * walsh_ep_combine: y [world * ntok, C], this rank's experts' outputs over
 * its received rows, back to the owners of the tokens: the columns of this
 * rank's experts of rows j * ntok .. into rank j's y_full; then flags[world
 * + rank] = epoch on rank j.
 * walsh_ep_wait: one small kernel waiting until flags[first .. first + n - 1]
 * all equal epoch, for at most timeout_cycles SM clock cycles; on expiry it
 * writes WALSH_ERR_TIMEOUT to *status (device int) and returns, so that the
 * host reads the failure at its next synchronisation.
 * The exchange kernels use plain 16-byte stores to peer memory and a system-
 * scope release of the flag (no TMA).  No counterpart in the
 * reference (its MoE runs on one device). */
walsh_status walsh_ep_dispatch(const void* u, int dtype, int64_t ntok, int C, const float* weights, int rank,
                               int world, void* const* peer_recv_u, float* const* peer_recv_w,
                               uint32_t* const* peer_flags, uint32_t* counters, uint32_t epoch, void* stream);
walsh_status walsh_ep_combine(const void* y, int dtype, int64_t ntok, int C, int rank, int world,
                              void* const* peer_y, uint32_t* const* peer_flags, uint32_t* counters,
                              uint32_t epoch, void* stream);
walsh_status walsh_ep_wait(const uint32_t* flags, int first, int n, uint32_t epoch, long long timeout_cycles,
                           int* status, void* stream);

/* CUDA IPC plumbing for the exchange buffers.  walsh_ipc_handle: the handle
 * (walsh_ipc_handle_bytes() bytes) of the allocation dev_ptr lies in, and
 * dev_ptr's byte offset in it (pooling allocators hand out sub-ranges).
 * walsh_ipc_open: the mapping of such a handle in another process (peer
 * access enabled on first use): *dev_ptr_out = base + offset, *base_out =
 * the mapping to pass to walsh_ipc_close.  No counterpart in the reference. */
walsh_status walsh_ipc_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out);
walsh_status walsh_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out, void** base_out);
walsh_status walsh_ipc_close(void* base);
int walsh_ipc_handle_bytes(void);

/* Ternary tensor of a .walsh v4 file ('B' chunk: bitmask + sign bits, as
 * compress.py:36-93 writes it and generate_compressed.py:70-105 reads it) to
 * dense float values (row-major, `total` = rows x k elements) and,
 * optionally (packed != NULL), this library's 2-bit layout [rows, ceil(k/4)]
 * for the last dimension k.  All pointers are device memory; mask_bytes and
 * sign_bytes are the chunk's array lengths.  A population count of the
 * bitmask different from num_nonzero sets *err = WALSH_ERR_ARG (device
 * int, read by the caller after synchronising).
 * Replaces unpack_bitmask_ternary (generate_compressed.py:70-105). */
walsh_status walsh_bitmask_ternary_unpack(const uint8_t* bitmask, int64_t mask_bytes, const uint8_t* sign_bits,
                                          int64_t sign_bytes, int64_t total, int64_t num_nonzero, int k,
                                          float* dense, uint8_t* packed, int* err, void* stream);

/* Rows row0 .. row0 + nrows - 1 of the hash-embedding matrix:
 * out[r, :] = scale * sum_t importance[v, t] * tables[t, indices[v, t], :],
 * v = row0 + r (tables float [num_tables, buckets, C], importance float
 * [V, num_tables], indices int64 [V, num_tables], out float [nrows, C]; C a
 * multiple of 4, tables and out 16-byte aligned).  An index outside
 * [0, buckets) is skipped and sets *err = WALSH_ERR_INDEX (device int).
 * Replaces HashEmbedding._get_chunk_embeddings (src/model/chassis.py:175-191),
 * which the forward, output_projection and chunked_cross_entropy use. */
walsh_status walsh_hash_embed_rows(const float* tables, int64_t buckets, const float* importance,
                                   const int64_t* indices, int num_tables, int C, float scale, int64_t row0,
                                   int64_t nrows, float* out, int* err, void* stream);

/* HadamardLinear(F, F), F = features = 512 or 2048, for 16-bit activations
 * reading the ternary weights in their 2-bit packed form: x, y [ntok, F]
 * (dtype WALSH_BF16 or WALSH_F16, 16-byte aligned), w_2bit [32, F/32, F/128]
 * (the reference encoding, 16-byte aligned), alpha, beta float [32, F/32];
 * weight scale 1 (the HadamardLinear semantics).  Transforms in float32 on
 * the CUDA cores, the ternary mat-vecs on the tensor cores with 16-bit
 * operands and float32 accumulation (F = 2048: mat-vec results rounded to
 * the 16-bit type before the output transform).  Other F: WALSH_ERR_SHAPE.
 * Replaces HadamardLinear.forward (src/model/fht_cuda.py:489-519). */
walsh_status walsh_hadamard_linear_pk_fwd(const void* x, int dtype, int64_t ntok, int features,
                                          const uint8_t* w_2bit, const float* alpha, const float* beta, void* y,
                                          void* stream);
/* HadamardLinear(F, F) as one dense matrix for the tensor-core GEMM form of
 * walsh_hadamard_linear_dense_fwd: from the 2-bit packed weights w_2bit
 * [32, F/32, F/128] and alpha, beta float [32, F/32] (F = features = 512 or
 * 2048) writes w_dense [F, F] in dtype (WALSH_BF16 or WALSH_F16) and scale
 * float [F] with scale[r] w_dense[r, c] = beta . H W H . alpha at (r, c), the
 * two normalised 32-point transforms included.  Each entry is an integer in
 * [-32, 32] times alpha[c] and a power of two, rounded once to the 16-bit
 * type.  Derived from HadamardLinear.forward (src/model/fht_cuda.py:489-519):
 * the reference has no such matrix; this is weight preparation, run once
 * per weight update. */
walsh_status walsh_hadamard_linear_dense_weights(const uint8_t* w_2bit, const float* alpha, const float* beta,
                                                 int features, int dtype, void* w_dense, float* scale,
                                                 void* stream);
/* HadamardLinear(F, F) for 16-bit activations as one tcgen05 GEMM over the
 * matrix of walsh_hadamard_linear_dense_weights: y[t, r] = scale[r] sum_c
 * x[t, c] w_dense[r, c], float32 accumulation, y rounded once to dtype.  x, y
 * [ntok, F] (16-byte aligned), w_dense [F, F] in x's dtype (16-byte aligned),
 * scale float [F] (16-byte aligned).  Replaces HadamardLinear.forward
 * (src/model/fht_cuda.py:489-519) where it is faster than the packed kernel
 * (F = 512 at thousands of tokens). */
walsh_status walsh_hadamard_linear_dense_fwd(const void* x, int dtype, int64_t ntok, int features,
                                             const void* w_dense, const float* scale, void* y, void* stream);
/* Status word of walsh_hadamard_linear_pk_fwd's bounded waits (0 or
 * WALSH_ERR_TIMEOUT); synchronous read, reset != 0 clears it. */
int walsh_hlin_pk_error(int reset);

/* ---------------------------------------------------------------------------
 * Dense helpers around the layer stack
 * ------------------------------------------------------------------------- */

/* Gather rows of a [V, D] table for token ids idx[ntok] (int64) into
 * out [ntok, D].  Ids outside [0, V) write zeros and set *err to
 * WALSH_ERR_INDEX (err may be NULL).
 * Replaces tok_embeddings (nn.Embedding) followed by stream_proj, whose
 * weights are folded into the table at load (src/model/mhc.py:634-640). */
walsh_status walsh_embed_gather(const int64_t* idx, int64_t ntok, const void* table, int dtype,
                                int64_t V, int D, void* out, int* err, void* stream);

/* y[m, n] = sum_k x[m*ldx + k] w[n, k] + bias[n] (bias may be NULL).
 * x, w, y each float32 or bfloat16.  Used for stream_merge, the tied output
 * projection and the load-time embedding/stream_proj fold
 * (src/model/mhc.py:654-676). */
walsh_status walsh_linear_fwd(const void* x, int x_dtype, int64_t M, int K, int64_t ldx,
                              const void* w, int w_dtype, int64_t N, const float* bias, void* y,
                              int y_dtype, void* stream);

/* walsh_linear_split_fwd for float32 x without bias on the 5th-generation
 * tensor cores: the three split products as one GEMM with K tripled,
 * [x_hi | x_hi | x_lo] w3^T with w3 [N, 3K] bfloat16 = [w_hi | w_lo | w_hi]
 * (rows 16-byte aligned: K % 8 == 0), fp32 accumulation, y float32 [M, N]
 * (any N).  scratch: walsh_linear_split_tc_scratch_bytes(M, K) bytes,
 * 16-byte aligned.  Same role as walsh_linear_split_fwd for the tied output
 * projection (src/model/mhc.py:654-676). */
int64_t walsh_linear_split_tc_scratch_bytes(int64_t M, int K);
walsh_status walsh_linear_split_tc_fwd(const float* x, int64_t M, int K, const void* w3, int64_t N,
                                       void* scratch, float* y, void* stream);

/* y[m, n] = sum_k x[m*ldx + k] w[n, k] + bias[n] in float32 on the tensor
 * cores, with w given as two bfloat16 matrices w_hi + w_lo (w_hi = bf16(w),
 * w_lo = bf16(w - w_hi)); a float32 or float16 x is split the same way, a
 * bfloat16 x is used as is.  x 16-byte aligned with ldx*size a multiple of
 * 16, K a multiple of 32, y float32 [M, N].  Accuracy about 2^-16 relative
 * per product.  Same role as walsh_linear_fwd for stream_merge and the tied
 * output projection (src/model/mhc.py:654-676). */
walsh_status walsh_linear_split_fwd(const void* x, int x_dtype, int64_t M, int K, int64_t ldx,
                                    const void* w_hi, const void* w_lo, int64_t N, const float* bias,
                                    float* y, void* stream);

/* Chassis RMSNorm: y = x / sqrt(mean(x^2) + eps) * w over rows of C.
 * Replaces RMSNorm.forward (src/model/chassis.py:96-106). */
walsh_status walsh_rmsnorm(const void* x, int dtype, int64_t rows, int C, const float* w,
                           float eps, void* y, int y_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WALSH_H_ */
