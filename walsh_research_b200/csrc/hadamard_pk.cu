// HadamardLinear for 16-bit activations with the ternary weights read in
// their 2-bit packed form: C_in = C_out = 512 (32 groups x 16) and
// C_in = C_out = 2048 (32 groups x 64).
//
// Per token (src/model/fht_cuda.py:489-519), with H the +-1 Sylvester matrix
// of order 32 (the reference's H is H / sqrt(32)):
//   Z[g][i] = sum_g' H[g][g'] alpha[g'][i] x[g'][i]          (transform A)
//   V[g][o] = sum_i  w[g][o][i] Z[g][i]                       (ternary mat-vecs)
//   y[h][o] = beta[h][o] / 32 * sum_g H[h][g] V[g][o]         (transform C)
//
// One persistent CTA of 16 warps per SM walks 64-token tiles.  Per tile:
//   A  thread (t, p) takes columns 2p, 2p + 1 of token t, read straight from
//      global memory (32 four-byte loads per thread; four tokens x 32 bytes
//      per warp access), scaled by alpha, transformed by in-register
//      butterflies on float pairs, rounded to the 16-bit type into shared
//      memory; the next tile's loads are then issued into the same registers,
//      so they arrive while this tile finishes;
//   B  warp w takes groups 2w, 2w + 1: m16n8k16 MMAs with A = the 64 tokens'
//      16-wide slice of group g (ldmatrix) and B = w_g^T, whose fragments
//      were built once from the 2-bit codes (the packed weights, 2 KB, are
//      staged with 128-bit loads); float32 results to shared memory;
//   C  thread (t, p): output columns 2p, 2p + 1 over the 32 groups, the
//      butterfly transform, beta / 32, rounded and written straight to
//      global memory.
// Rows are padded in shared memory (16-bit rows by 16 bytes, float32 rows by
// 32 bytes) and a warp takes every other token of eight in A and C, so that
// a warp's accesses (ldmatrix rows included) fall in distinct banks.  The kernel
// has no waits besides block barriers (walsh_hlin_pk_error stays 0; it is
// kept for the status interface of the entry point).
#include <type_traits>

#include "common.cuh"
#include "mma.cuh"
#include "tc05.cuh"

namespace walsh {

__device__ int g_hlin_pk_error;

template <typename T16>
__device__ __forceinline__ uint32_t ternary_pair16(int a, int b) {
  // (a, b) in {-1, 0, 1} as a 16-bit pair (a in the low half)
  const uint16_t one = std::is_same<T16, __half>::value ? 0x3C00u : 0x3F80u;
  const uint16_t va = a == 0 ? 0 : (uint16_t)(one | (a < 0 ? 0x8000u : 0u));
  const uint16_t vb = b == 0 ? 0 : (uint16_t)(one | (b < 0 ? 0x8000u : 0u));
  return (uint32_t)va | ((uint32_t)vb << 16);
}

namespace hpk2 {
constexpr int C = 512, G = 32, IO = 16, TM = 64, NW = 16, NT = NW * 32;
constexpr int ZROW = C * 2 + 16;       // bytes per token of the transformed input (16-bit)
constexpr int VROW = G * IO * 4 + 32;  // bytes per token of the mat-vec results (float32)
constexpr int WBYTES = G * IO * IO / 4;  // packed weights
constexpr int OFF_V = TM * ZROW, OFF_AB = OFF_V + TM * VROW, OFF_W = OFF_AB + 2 * G * IO * 4;
constexpr int SMEM = OFF_W + WBYTES + 128;
}  // namespace hpk2

__device__ __forceinline__ uint64_t hpk_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 hpk_unpack(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(lo), "=f"(hi) : "l"(v));
  return make_float2(lo, hi);
}
__device__ __forceinline__ uint64_t hpk_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t hpk_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t hpk_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// unnormalised 32-point Walsh-Hadamard transform of 32 float pairs (Sylvester order)
__device__ __forceinline__ void fht32x2(uint64_t* v) {
#pragma unroll
  for (int s = 1; s < 32; s <<= 1)
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if ((i & s) == 0) {
        const uint64_t a = v[i], b = v[i + s];
        v[i] = hpk_add(a, b);
        v[i + s] = hpk_sub(a, b);
      }
}

template <typename T16>
__global__ void __launch_bounds__(hpk2::NT, 1)
hlin_packed_kernel(const T16* __restrict__ x, int64_t ntok, const uint8_t* __restrict__ w2,
                   const float* __restrict__ alpha, const float* __restrict__ beta, T16* __restrict__ y) {
  using namespace hpk2;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, t4 = lane & 3;
  const int64_t ntiles = (ntok + TM - 1) / TM;
  // packed weights (16 bytes per thread), alpha and beta / 32 into shared memory
  if (tid < WBYTES / 16)
    reinterpret_cast<uint4*>(sm + OFF_W)[tid] = __ldg(reinterpret_cast<const uint4*>(w2) + tid);
  float* ab = reinterpret_cast<float*>(sm + OFF_AB);  // [G][IO] alpha, then [G][IO] beta / 32
  for (int q = tid; q < G * IO; q += NT) {
    ab[q] = __ldg(alpha + q);
    ab[G * IO + q] = __ldg(beta + q) * (1.0f / 32.0f);
  }
  __syncthreads();
  // B fragments of w_g^T for this warp's groups 2w, 2w + 1 (n-tiles: o 0-7, 8-15)
  uint32_t bf[2][2][2];
  {
    const uint8_t* ws = sm + OFF_W;
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int g = 2 * warp + q, o = 8 * nt + gid, i0 = 8 * h + 2 * t4;
          const uint32_t byte = ws[(g * IO + o) * 4 + (i0 >> 2)];
          const int s0 = 6 - 2 * (i0 & 3);
          const int a = (int)((byte >> s0) & 3u) - 1, b = (int)((byte >> (s0 - 2)) & 3u) - 1;
          bf[q][nt][h] = ternary_pair16<T16>(a, b);
        }
  }
  // token row and first column of this thread in A and C: a warp's four
  // tokens are b, b + 2, b + 4, b + 6 (b = 8 (w / 2) + w % 2), so that its
  // 16-bit row pieces (rows 4 banks apart) and the float32 pairs each half
  // warp reads in C (rows 8 banks apart) fall in distinct banks
  const int trow = ((warp >> 1) << 3) | (warp & 1) | ((lane >> 3) << 1), pc = (lane & 7) * 2;
  const uint64_t* ab2 = reinterpret_cast<const uint64_t*>(ab);
  uint32_t xr[G];  // this thread's two input columns of its token, 16-bit pairs
  auto load_x = [&](int64_t tile) {
    const int64_t tok = tile * TM + trow;
    if (tile < ntiles && tok < ntok) {
      const uint32_t* xp = reinterpret_cast<const uint32_t*>(x + tok * C + pc);
#pragma unroll
      for (int g = 0; g < G; ++g) xr[g] = __ldg(xp + g * (IO / 2));
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) xr[g] = 0u;
    }
  };
  load_x(blockIdx.x);
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t tok = tile * TM + trow;
    // ---- A
    {
      uint64_t v[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 f = unpack2<T16>(xr[g]);
        v[g] = hpk_mul(hpk_pack(f.x, f.y), ab2[(g * IO + pc) / 2]);
      }
      load_x(tile + gridDim.x);  // next tile's columns, in flight during B and C
      fht32x2(v);
      unsigned char* zp = sm + trow * ZROW + pc * 2;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 f = hpk_unpack(v[g]);
        *reinterpret_cast<uint32_t*>(zp + g * IO * 2) = pack2<T16>(f.x, f.y);
      }
    }
    __syncthreads();
    // ---- B: the ternary mat-vecs of groups 2w, 2w + 1 on the tensor cores
    {
      const uint32_t zs = tc05::smem_u32(sm);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int g = 2 * warp + q;
#pragma unroll
        for (int mt = 0; mt < TM / 16; ++mt) {
          uint32_t a[4];
          const uint32_t addr = zs + (uint32_t)((16 * mt + (lane & 15)) * ZROW + g * IO * 2 + (lane >> 4) * 16);
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                       : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                       : "r"(addr));
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            mma16<T16>(c, a, bf[q][nt][0], bf[q][nt][1]);
            const int t0 = 16 * mt + gid, o = 8 * nt + 2 * t4;
            *reinterpret_cast<float2*>(sm + OFF_V + t0 * VROW + (g * IO + o) * 4) = make_float2(c[0], c[1]);
            *reinterpret_cast<float2*>(sm + OFF_V + (t0 + 8) * VROW + (g * IO + o) * 4) = make_float2(c[2], c[3]);
          }
        }
      }
    }
    __syncthreads();
    // ---- C: output columns pc, pc + 1 of token trow over the 32 groups, to global memory
    {
      const unsigned char* vp = sm + OFF_V + trow * VROW + pc * 4;
      uint64_t v[G];
#pragma unroll
      for (int g = 0; g < G; ++g) v[g] = *reinterpret_cast<const uint64_t*>(vp + g * IO * 4);
      fht32x2(v);
      if (tok < ntok) {
        uint32_t* yp = reinterpret_cast<uint32_t*>(y + tok * C + pc);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float2 f = hpk_unpack(hpk_mul(v[h], ab2[(G * IO + h * IO + pc) / 2]));
          yp[h * (IO / 2)] = pack2<T16>(f.x, f.y);
        }
      }
    }
    __syncthreads();  // Z and V are free for the next tile
  }
}

// ---------------------------------------------------------------------------
// C = 2048 (32 groups x 64).  One persistent CTA of 16 warps per SM walks
// 32-token tiles (16-token tiles while there are at most as many as SMs) through
// one buffer of 32 (16) rows (the 16-bit transformed input, then in place
// the 16-bit mat-vec results):
//   A  warp t takes tokens t and 16 + t of the tile, lane p its columns 2p, 2p + 1 in
//      each group (one 128-byte line per warp load), scaled by alpha,
//      butterfly-transformed on float pairs, rounded into the row; the next
//      tile's columns are then loaded into the same registers;
//   B  warp w takes groups 2w, 2w + 1: A = the two 16 x 64 blocks of group g
//      (ldmatrix, all k-steps held before the blocks are overwritten),
//      B = w_g^T, 32 fragments per group (each used by both blocks' MMAs) decoded from this lane's 2-bit
//      codes (8 words per group, re-laid in shared memory once per CTA:
//      code pairs at bits 2r and 2r + 16, decoded as the 16-bit integers
//      1024 + c (fp16) or 128 + c (bf16) less 1025 or 129, exact); each
//      16 x 8 result is rounded to the 16-bit type and written over its own
//      columns of the block;
//   C  warp t, lane p: its two tokens' output columns 2p, 2p + 1 over the 32 groups, the
//      butterfly transform, beta / 32, written straight to global memory.
// Row pitch 4112 bytes: ldmatrix rows and fragment stores fall in distinct
// banks; the A and C accesses of a warp are one contiguous 128-byte row
// piece.  A thread's C reads and its next A writes touch the same elements,
// so a tile needs two block barriers.
// ---------------------------------------------------------------------------
namespace hpk4 {
constexpr int C = 2048, G = 32, IO = 64, TS = 16, NW = 16, NT = NW * 32;
constexpr int ZROW = C * 2 + 16;
// tiles of NH 16-token halves (NH = 2 from a wave of 32-token tiles on; 1 below)
template <int NH>
struct Lay {
  static constexpr int TM = NH * TS;
  static constexpr int OFF_AB = TM * ZROW;
  static constexpr int OFF_W = OFF_AB + 2 * G * IO * 4;  // [2 groups][8 n-tiles][NT threads] code words
  static constexpr int SMEM = OFF_W + 16 * NT * 4;
};
}  // namespace hpk4

template <typename T16>
__device__ __forceinline__ uint32_t ternary_code_pair(uint32_t word, int r) {
  // code pair r of a register word (codes at bits 2r and 2r + 16) as the
  // 16-bit pair (c_lo - 1, c_hi - 1)
  if constexpr (std::is_same<T16, __half>::value) {
    const uint32_t v = ((word >> (2 * r)) & 0x00030003u) | 0x64006400u;  // 1024 + c
    __half2 h;
    memcpy(&h, &v, 4);
    h = __hsub2(h, __float2half2_rn(1025.0f));
    uint32_t o;
    memcpy(&o, &h, 4);
    return o;
  } else {
    const uint32_t v = ((word >> (2 * r)) & 0x00030003u) | 0x43004300u;  // 128 + c
    __nv_bfloat162 h;
    memcpy(&h, &v, 4);
    h = __hsub2(h, __float2bfloat162_rn(129.0f));
    uint32_t o;
    memcpy(&o, &h, 4);
    return o;
  }
}

template <typename T16, int NH>
__global__ void __launch_bounds__(hpk4::NT, 1)
hlin_packed2048_kernel(const T16* __restrict__ x, int64_t ntok, const uint8_t* __restrict__ w2,
                       const float* __restrict__ alpha, const float* __restrict__ beta, T16* __restrict__ y) {
  using namespace hpk4;
  constexpr int TM = Lay<NH>::TM, OFF_AB = Lay<NH>::OFF_AB, OFF_W = Lay<NH>::OFF_W;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, t4 = lane & 3;
  const int64_t ntiles = (ntok + TM - 1) / TM;  // tiles of NH 16-token halves
  float* ab = reinterpret_cast<float*>(sm + OFF_AB);  // [G][IO] alpha, then [G][IO] beta / 32
  for (int q = tid; q < G * IO; q += NT) {
    ab[q] = __ldg(alpha + q);
    ab[G * IO + q] = __ldg(beta + q) * (1.0f / 32.0f);
  }
  // this lane's codes of w_g^T for groups 2w, 2w + 1: word [q][nt] holds the
  // pairs r = 2 ks + h (k rows 16 ks + 8 h + 2 t4, + 1; column 8 nt + gid)
  uint32_t* wpk = reinterpret_cast<uint32_t*>(sm + OFF_W);
#pragma unroll 1
  for (int q = 0; q < 2; ++q)
#pragma unroll 1
    for (int nt = 0; nt < 8; ++nt) {
      const int g = 2 * warp + q, o = 8 * nt + gid;
      const uint8_t* row = w2 + (g * IO + o) * (IO / 4);
      uint32_t wd = 0;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int i0 = 8 * r + 2 * t4;  // = 16 ks + 8 h + 2 t4
        const uint32_t byte = __ldg(row + (i0 >> 2));
        const int s0 = 6 - 2 * (i0 & 3);
        wd |= ((byte >> s0) & 3u) << (2 * r);
        wd |= ((byte >> (s0 - 2)) & 3u) << (2 * r + 16);
      }
      wpk[(q * 8 + nt) * NT + tid] = wd;
    }
  __syncthreads();
  const int pc = 2 * lane;  // columns of this lane in A and C (token = warp)
  const uint64_t* ab2 = reinterpret_cast<const uint64_t*>(ab);
  uint32_t xr[G];
  // token row `half` (0 .. NH - 1) of tile `tile` for this warp
  auto load_x = [&](int64_t tile, int half) {
    const int64_t tok = tile * TM + half * TS + warp;
    if (tile < ntiles && tok < ntok) {
      const uint32_t* xp = reinterpret_cast<const uint32_t*>(x + tok * C + pc);
#pragma unroll
      for (int g = 0; g < G; ++g) xr[g] = __ldg(xp + g * (IO / 2));
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) xr[g] = 0u;
    }
  };
  load_x(blockIdx.x, 0);
  const uint32_t zs = tc05::smem_u32(sm);
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    // ---- A, for tokens warp (and 16 + warp) of the tile
#pragma unroll 1
    for (int half = 0; half < NH; ++half) {
      unsigned char* zrow = sm + (half * TS + warp) * ZROW + pc * 2;
      uint64_t v[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 f = unpack2<T16>(xr[g]);
        v[g] = hpk_mul(hpk_pack(f.x, f.y), ab2[(g * IO + pc) / 2]);
      }
      if (half + 1 < NH)
        load_x(tile, half + 1);
      else
        load_x(tile + gridDim.x, 0);
      fht32x2(v);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 f = hpk_unpack(v[g]);
        *reinterpret_cast<uint32_t*>(zrow + g * IO * 2) = pack2<T16>(f.x, f.y);
      }
    }
    __syncthreads();
    // ---- B: groups 2w, 2w + 1 over the NH 16-row halves (each decoded B
    // fragment serves NH MMAs), results over their own block
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      const int g = 2 * warp + q;
      uint32_t a[NH][4][4];
#pragma unroll
      for (int mt = 0; mt < NH; ++mt)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t addr =
              zs + (uint32_t)((mt * TS + (lane & 15)) * ZROW + (g * IO + ks * 16 + (lane >> 4) * 8) * 2);
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                       : "=r"(a[mt][ks][0]), "=r"(a[mt][ks][1]), "=r"(a[mt][ks][2]), "=r"(a[mt][ks][3])
                       : "r"(addr)
                       : "memory");
        }
      __syncwarp();
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const uint32_t wd = wpk[(q * 8 + nt) * NT + tid];
        float cc[NH][4];
#pragma unroll
        for (int mt = 0; mt < NH; ++mt) cc[mt][0] = cc[mt][1] = cc[mt][2] = cc[mt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t b0 = ternary_code_pair<T16>(wd, 2 * ks), b1 = ternary_code_pair<T16>(wd, 2 * ks + 1);
#pragma unroll
          for (int mt = 0; mt < NH; ++mt) mma16<T16>(cc[mt], a[mt][ks], b0, b1);
        }
        unsigned char* vp = sm + gid * ZROW + (g * IO + 8 * nt + 2 * t4) * 2;
#pragma unroll
        for (int mt = 0; mt < NH; ++mt) {
          *reinterpret_cast<uint32_t*>(vp + mt * TS * ZROW) = pack2<T16>(cc[mt][0], cc[mt][1]);
          *reinterpret_cast<uint32_t*>(vp + (mt * TS + 8) * ZROW) = pack2<T16>(cc[mt][2], cc[mt][3]);
        }
      }
    }
    __syncthreads();
    // ---- C: output columns pc, pc + 1 of this warp's tokens over the 32 groups
#pragma unroll 1
    for (int half = 0; half < NH; ++half) {
      const int64_t tok = tile * TM + half * TS + warp;
      const unsigned char* zrow = sm + (half * TS + warp) * ZROW + pc * 2;
      uint64_t v[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 f = unpack2<T16>(*reinterpret_cast<const uint32_t*>(zrow + g * IO * 2));
        v[g] = hpk_pack(f.x, f.y);
      }
      fht32x2(v);
      if (tok < ntok) {
        uint32_t* yp = reinterpret_cast<uint32_t*>(y + tok * C + pc);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float2 f = hpk_unpack(hpk_mul(v[h], ab2[(G * IO + h * IO + pc) / 2]));
          yp[h * (IO / 2)] = pack2<T16>(f.x, f.y);
        }
      }
    }
    // the next tile's A writes only the elements this thread just read
  }
}

static int hlin_pk_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      n = 148;
    }
  }
  return n;
}

}  // namespace walsh

using namespace walsh;

template <typename T16>
static int launch_hlin_pk2048(const void* x, int64_t ntok, const uint8_t* w2, const float* alpha, const float* beta,
                              void* y, cudaStream_t s) {
  // 32-token tiles (each decoded weight fragment serves two 16-token MMAs)
  // once 16-token tiles would give a CTA more than one (4096 tokens: 20.1
  // against 22.1 us); 16-token tiles below, for more CTAs (64 tokens: 13.7
  // against 18.4 us)
  const int sms = hlin_pk_sms();
  if ((ntok + 15) / 16 > sms) {
    using L = hpk4::Lay<2>;
    const int64_t ntiles = (ntok + L::TM - 1) / L::TM;
    const int grid = (int)min64(ntiles, sms);
    auto k = hlin_packed2048_kernel<T16, 2>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM) != cudaSuccess)
      return launch_status();
    k<<<grid, hpk4::NT, L::SMEM, s>>>((const T16*)x, ntok, w2, alpha, beta, (T16*)y);
    return launch_status();
  }
  using L = hpk4::Lay<1>;
  const int64_t ntiles = (ntok + L::TM - 1) / L::TM;
  const int grid = (int)min64(ntiles, sms);
  auto k = hlin_packed2048_kernel<T16, 1>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM) != cudaSuccess)
    return launch_status();
  k<<<grid, hpk4::NT, L::SMEM, s>>>((const T16*)x, ntok, w2, alpha, beta, (T16*)y);
  return launch_status();
}

// HadamardLinear(F, F) as one matrix for the dense tensor-core form:
// out row r = (h, o), column c = (p, i), with the unnormalised Sylvester
// matrix H[a, b] = (-1)^popcount(a & b):
//   w_dense[r, c] = alpha[p, i] sum_g H[g, h] H[p, g] w[g, o, i] / (32 q),
//   scale[r]      = beta[h, o] q,
// so that y = scale . (x w_dense^T) equals beta . H W H (alpha . x) with the
// reference's normalised transforms (HadamardLinear.forward,
// src/model/fht_cuda.py:489-519).  The 32-term sum is an integer in
// [-32, 32]; q is the power of two at or above max |alpha|, which keeps
// every entry at most 1 in magnitude (float16 range).  One block per row.
template <typename T16>
__global__ void __launch_bounds__(256) hlin_dense_prep_kernel(const uint8_t* __restrict__ w2,
                                                              const float* __restrict__ alpha,
                                                              const float* __restrict__ beta, int io,
                                                              T16* __restrict__ wd, float* __restrict__ scale) {
  __shared__ float red[8];
  const int F = 32 * io, row = blockIdx.x, h = row / io, o = row % io, kb = (io + 3) / 4;
  float a = 0.f;
  for (int c = threadIdx.x; c < F; c += blockDim.x) a = fmaxf(a, fabsf(__ldg(alpha + c)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  a = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) a = fmaxf(a, red[w]);
  int e = 0;
  if (a > 0.f && a <= 3.0e38f) frexpf(a, &e);  // a = m 2^e, m in [0.5, 1)
  const float q = ldexpf(1.f, e), inv = ldexpf(1.f, -e - 5);
  if (threadIdx.x == 0) scale[row] = __ldg(beta + row) * q;
  for (int c = threadIdx.x; c < F; c += blockDim.x) {
    const int p = c / io, i = c % io;
    int sum = 0;
#pragma unroll 8
    for (int g = 0; g < 32; ++g) {
      const int v = (int)((__ldg(w2 + ((size_t)g * io + o) * kb + (i >> 2)) >> (6 - 2 * (i & 3))) & 3u) - 1;
      sum += ((__popc(g & h) + __popc(p & g)) & 1) ? -v : v;
    }
    wd[(size_t)row * F + c] = from_f<T16>((float)sum * __ldg(alpha + c) * inv);
  }
}

extern "C" walsh_status walsh_hadamard_linear_dense_weights(const uint8_t* w_2bit, const float* alpha,
                                                            const float* beta, int features, int dtype,
                                                            void* w_dense, float* scale, void* stream) {
  if (int e = injected("hadamard_linear_dense_weights")) return e;
  WALSH_CHECK_ARG(w_2bit && alpha && beta && w_dense && scale);
  WALSH_CHECK_SHAPE(features == 512 || features == 2048);
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  cudaStream_t s = (cudaStream_t)stream;
  const int io = features / 32;
  if (dtype == WALSH_BF16)
    hlin_dense_prep_kernel<__nv_bfloat16><<<features, 256, 0, s>>>(w_2bit, alpha, beta, io,
                                                                   (__nv_bfloat16*)w_dense, scale);
  else
    hlin_dense_prep_kernel<__half><<<features, 256, 0, s>>>(w_2bit, alpha, beta, io, (__half*)w_dense, scale);
  return launch_status();
}

extern "C" walsh_status walsh_hadamard_linear_pk_fwd(const void* x, int dtype, int64_t ntok, int features,
                                                     const uint8_t* w_2bit, const float* alpha, const float* beta,
                                                     void* y, void* stream) {
  if (int e = injected("hadamard_linear_pk_fwd")) return e;
  WALSH_CHECK_ARG(x && w_2bit && alpha && beta && y);
  WALSH_CHECK_SHAPE(ntok >= 0 && (features == 512 || features == 2048));
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  if ((((uintptr_t)x) | ((uintptr_t)y) | ((uintptr_t)w_2bit)) & 15u) return WALSH_ERR_ALIGN;
  if (ntok == 0) return WALSH_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (features == 2048)
    return dtype == WALSH_BF16 ? launch_hlin_pk2048<__nv_bfloat16>(x, ntok, w_2bit, alpha, beta, y, s)
                               : launch_hlin_pk2048<__half>(x, ntok, w_2bit, alpha, beta, y, s);
  const int64_t ntiles = (ntok + hpk2::TM - 1) / hpk2::TM;
  const int grid = (int)min64(ntiles, hlin_pk_sms());
  if (dtype == WALSH_BF16) {
    auto k = hlin_packed_kernel<__nv_bfloat16>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, hpk2::SMEM) != cudaSuccess)
      return launch_status();
    k<<<grid, hpk2::NT, hpk2::SMEM, s>>>((const __nv_bfloat16*)x, ntok, w_2bit, alpha, beta, (__nv_bfloat16*)y);
  } else {
    auto k = hlin_packed_kernel<__half>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, hpk2::SMEM) != cudaSuccess)
      return launch_status();
    k<<<grid, hpk2::NT, hpk2::SMEM, s>>>((const __half*)x, ntok, w_2bit, alpha, beta, (__half*)y);
  }
  return launch_status();
}

extern "C" int walsh_hlin_pk_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_hlin_pk_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_hlin_pk_error, &zero, sizeof(int));
  }
  return v;
}
