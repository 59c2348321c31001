// Hash embeddings (HashEmbedding, src/model/chassis.py:109-260): token v's
// embedding is sqrt(C) * sum_i importance[v, i] * table_i[index[v, i]], with
// index[v, i] = ((a_i v + b_i) mod p) mod buckets precomputed per vocabulary
// entry.  The forward gathers it per token, and the output projection and
// the chunked cross entropy contract hidden states with it for every
// vocabulary row; both reduce to the same [V, C] matrix, which this kernel
// builds for a range of rows (the model caches it with the other derived
// weights, so embedding lookups and logits then run on the dense paths).
#include "common.cuh"

namespace walsh {

// One thread per (row, 4 columns); tables are [nt][buckets][C] float32.
__global__ void hash_embed_rows_kernel(const float* __restrict__ tables, int64_t buckets,
                                       const float* __restrict__ importance, const int64_t* __restrict__ indices,
                                       int nt, int C, float scale, int64_t row0, int64_t nrows, float* __restrict__ out,
                                       int* __restrict__ err) {
  const int c4 = C / 4;
  const int64_t total = nrows * c4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / c4;
    const int c = (int)(i - r * c4) * 4;
    const int64_t v = row0 + r;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < nt; ++t) {
      const int64_t b = indices[v * nt + t];
      if (b < 0 || b >= buckets) {
        atomicExch(err, (int)WALSH_ERR_INDEX);
        continue;
      }
      const float w = importance[v * nt + t];
      const float4 e = *reinterpret_cast<const float4*>(tables + ((int64_t)t * buckets + b) * C + c);
      // sum over tables in order, product then sum (no fused multiply-add),
      // as the reference's per-table accumulation rounds
      acc.x = __fadd_rn(acc.x, __fmul_rn(e.x, w));
      acc.y = __fadd_rn(acc.y, __fmul_rn(e.y, w));
      acc.z = __fadd_rn(acc.z, __fmul_rn(e.z, w));
      acc.w = __fadd_rn(acc.w, __fmul_rn(e.w, w));
    }
    *reinterpret_cast<float4*>(out + r * C + c) =
        make_float4(__fmul_rn(acc.x, scale), __fmul_rn(acc.y, scale), __fmul_rn(acc.z, scale),
                    __fmul_rn(acc.w, scale));
  }
}

}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_hash_embed_rows(const float* tables, int64_t buckets, const float* importance,
                                              const int64_t* indices, int num_tables, int C, float scale,
                                              int64_t row0, int64_t nrows, float* out, int* err, void* stream) {
  if (int e = injected("hash_embed_rows")) return e;
  WALSH_CHECK_ARG(tables && importance && indices && out && err);
  WALSH_CHECK_SHAPE(buckets > 0 && num_tables >= 1 && C > 0 && C % 4 == 0 && row0 >= 0 && nrows >= 0);
  if ((((uintptr_t)tables) | ((uintptr_t)out)) & 15u) return WALSH_ERR_ALIGN;
  if (nrows == 0) return WALSH_OK;
  const int64_t total = nrows * (C / 4);
  int64_t g = (total + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  hash_embed_rows_kernel<<<(unsigned)g, 256, 0, (cudaStream_t)stream>>>(tables, buckets, importance, indices,
                                                                       num_tables, C, scale, row0, nrows, out, err);
  return launch_status();
}
