// Expert-parallel exchange of the Hadamard MoE over NVLink.
//
// Expert e of HadamardMoE consumes exactly feature block e (columns 32e ..
// 32e + 31) of a token and writes exactly that block of the output
// (src/model/moe.py:536-541), so expert parallelism is a transpose of the
// [tokens x blocks] matrix.  Ownership is in contiguous ranges: rank j of G
// owns experts [j E/G, (j + 1) E/G).
//
// Each rank holds, in memory its peers can address (CUDA IPC mappings):
//   recv_u [G * T, C]  row r * T + t: token t of rank r (only the columns of
//                      this rank's experts are written);
//   recv_w [G * T, E]  routing weights of those rows, zero outside this
//                      rank's experts;
//   y_full [T, C]      the MoE output of this rank's own tokens, each block
//                      written by the rank that owns the expert;
//   flags  [2 G]       u32: flags[r] = epoch once rank r's dispatch rows are
//                      in, flags[G + j] = epoch once owner j's outputs are in.
// The exchange kernels write straight into the peers' buffers with 16-byte
// stores over NVLink; the last CTA to finish a destination (a local arrival
// counter) fences at system scope and releases that destination's flag.  No
// kernel waits on another kernel of the same GPU.  The waits on peers are a
// separate one-CTA kernel with a clock budget: on expiry it records
// WALSH_ERR_TIMEOUT in the caller's status word and returns.  The data moves
// by plain stores only (no TMA).
#include <cuda.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace walsh {
namespace ep {

constexpr int kMaxRanks = 8;

struct Peers {
  void* p[kMaxRanks];
};
struct PeerFlags {
  uint32_t* p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// After a CTA's stores to destination `dst`: the last CTA of that destination
// (counted in counters[dst], reset for the next exchange) publishes `epoch`
// at flag_ptr.  Called by all threads of the CTA.
__device__ __forceinline__ void finish_dst(uint32_t* counters, int dst, uint32_t nblocks, uint32_t* flag_ptr,
                                           uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t done = atomicAdd(counters + dst, 1u) + 1u;
    if (done == nblocks) {
      counters[dst] = 0u;
      __threadfence_system();
      st_release_sys(flag_ptr, epoch);
    }
  }
}

// Dispatch: block (x, dst) copies tokens [x * TPB, ...) of this rank to rank
// dst: the u columns of dst's experts (16-bit, 8 per 16-byte chunk) and the
// routing-weight row with zeros outside dst's experts.
template <int TPB>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const uint4* __restrict__ u, const float* __restrict__ w,
                                                         int64_t ntok, int C, int E, int rank, int world, Peers pu,
                                                         Peers pw, PeerFlags pf, uint32_t* counters, uint32_t epoch) {
  const int dst = blockIdx.y;
  const int epr = E / world;                      // experts per rank
  const int cols = epr * 32, ch_row = cols / 8;   // 16-byte chunks per token row for dst
  const int c0 = dst * cols;
  const int64_t t0 = (int64_t)blockIdx.x * TPB;
  const int ntile = (int)min64(TPB, ntok - t0);
  uint4* du = reinterpret_cast<uint4*>(pu.p[dst]);
  float* dw = reinterpret_cast<float*>(pw.p[dst]);
  const int64_t row0 = (int64_t)rank * ntok + t0;  // destination row of token t0
  for (int i = threadIdx.x; i < ntile * ch_row; i += blockDim.x) {
    const int t = i / ch_row, c = i - t * ch_row;
    du[((row0 + t) * C + c0) / 8 + c] = u[((t0 + t) * C + c0) / 8 + c];
  }
  for (int i = threadIdx.x; i < ntile * E; i += blockDim.x) {
    const int t = i / E, e = i - t * E;
    const bool own = e >= dst * epr && e < (dst + 1) * epr;
    dw[(row0 + t) * E + e] = own ? w[(t0 + t) * E + e] : 0.f;
  }
  finish_dst(counters, dst, gridDim.x, pf.p[dst] + rank, epoch);
}

// Combine: block (x, dst) returns to rank dst the outputs of this rank's
// experts for dst's tokens [x * TPB, ...): rows dst * T + t of y (this rank's
// expert output over the received rows) into dst's y_full row t.
template <int TPB>
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint4* __restrict__ y, int64_t ntok, int C, int E,
                                                        int rank, int world, Peers py, PeerFlags pf,
                                                        uint32_t* counters, uint32_t epoch) {
  const int dst = blockIdx.y;
  const int epr = E / world;
  const int cols = epr * 32, ch_row = cols / 8;
  const int c0 = rank * cols;
  const int64_t t0 = (int64_t)blockIdx.x * TPB;
  const int ntile = (int)min64(TPB, ntok - t0);
  uint4* dy = reinterpret_cast<uint4*>(py.p[dst]);
  const int64_t src0 = (int64_t)dst * ntok + t0;
  for (int i = threadIdx.x; i < ntile * ch_row; i += blockDim.x) {
    const int t = i / ch_row, c = i - t * ch_row;
    dy[((t0 + t) * C + c0) / 8 + c] = y[((src0 + t) * C + c0) / 8 + c];
  }
  finish_dst(counters + world, dst, gridDim.x, pf.p[dst] + world + rank, epoch);
}

// Thread i < n waits until flags[first + i] == epoch, for at most `budget`
// SM clock cycles; on expiry *status = WALSH_ERR_TIMEOUT.
__global__ void ep_wait_kernel(const uint32_t* flags, int first, int n, uint32_t epoch, long long budget,
                               int* status) {
  const int i = threadIdx.x;
  if (i >= n) return;
  const uint32_t* f = flags + first + i;
  const long long t0 = clock64();
  while (ld_acquire_sys(f) != epoch) {
    if (clock64() - t0 > budget) {
      atomicExch(status, (int)WALSH_ERR_TIMEOUT);
      return;
    }
    __nanosleep(200);
  }
}

constexpr int kTPB = 16;  // tokens per CTA of the exchange kernels

static bool shape_ok(int64_t ntok, int C, int E, int world, int rank) {
  return ntok > 0 && world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world && C == 32 * E &&
         E % world == 0 && ((E / world) * 32) % 8 == 0 && ntok <= (int64_t)1 << 40;
}

}  // namespace ep
}  // namespace walsh

using namespace walsh;

extern "C" walsh_status walsh_ep_dispatch(const void* u, int dtype, int64_t ntok, int C, const float* weights,
                                          int rank, int world, void* const* peer_recv_u,
                                          float* const* peer_recv_w, uint32_t* const* peer_flags,
                                          uint32_t* counters, uint32_t epoch, void* stream) {
  if (int e = injected("ep_dispatch")) return e;
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  WALSH_CHECK_ARG(u && weights && peer_recv_u && peer_recv_w && peer_flags && counters && epoch != 0);
  const int E = C / 32;
  WALSH_CHECK_SHAPE(ep::shape_ok(ntok, C, E, world, rank));
  ep::Peers pu{}, pw{};
  ep::PeerFlags pf{};
  for (int j = 0; j < world; ++j) {
    WALSH_CHECK_ARG(peer_recv_u[j] && peer_recv_w[j] && peer_flags[j]);
    if ((((uintptr_t)peer_recv_u[j]) & 15u) || (((uintptr_t)peer_recv_w[j]) & 3u)) return WALSH_ERR_ALIGN;
    pu.p[j] = peer_recv_u[j];
    pw.p[j] = peer_recv_w[j];
    pf.p[j] = peer_flags[j];
  }
  if (((uintptr_t)u) & 15u) return WALSH_ERR_ALIGN;
  const dim3 grid((unsigned)((ntok + ep::kTPB - 1) / ep::kTPB), (unsigned)world);
  ep::ep_dispatch_kernel<ep::kTPB><<<grid, 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)u, weights, ntok, C, E, rank, world, pu, pw, pf, counters, epoch);
  return launch_status();
}

extern "C" walsh_status walsh_ep_combine(const void* y, int dtype, int64_t ntok, int C, int rank, int world,
                                         void* const* peer_y, uint32_t* const* peer_flags, uint32_t* counters,
                                         uint32_t epoch, void* stream) {
  if (int e = injected("ep_combine")) return e;
  if (dtype != WALSH_BF16 && dtype != WALSH_F16) return WALSH_ERR_DTYPE;
  WALSH_CHECK_ARG(y && peer_y && peer_flags && counters && epoch != 0);
  const int E = C / 32;
  WALSH_CHECK_SHAPE(ep::shape_ok(ntok, C, E, world, rank));
  ep::Peers py{};
  ep::PeerFlags pf{};
  for (int j = 0; j < world; ++j) {
    WALSH_CHECK_ARG(peer_y[j] && peer_flags[j]);
    if (((uintptr_t)peer_y[j]) & 15u) return WALSH_ERR_ALIGN;
    py.p[j] = peer_y[j];
    pf.p[j] = peer_flags[j];
  }
  if (((uintptr_t)y) & 15u) return WALSH_ERR_ALIGN;
  const dim3 grid((unsigned)((ntok + ep::kTPB - 1) / ep::kTPB), (unsigned)world);
  ep::ep_combine_kernel<ep::kTPB><<<grid, 256, 0, (cudaStream_t)stream>>>((const uint4*)y, ntok, C, E, rank, world,
                                                                          py, pf, counters, epoch);
  return launch_status();
}

extern "C" walsh_status walsh_ep_wait(const uint32_t* flags, int first, int n, uint32_t epoch,
                                      long long timeout_cycles, int* status, void* stream) {
  if (int e = injected("ep_wait")) return e;
  WALSH_CHECK_ARG(flags && status && epoch != 0 && timeout_cycles > 0);
  WALSH_CHECK_SHAPE(first >= 0 && n >= 1 && n <= 2 * ep::kMaxRanks);
  ep::ep_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flags, first, n, epoch, timeout_cycles, status);
  return launch_status();
}

// cuMemGetAddressRange through the runtime's driver entry point (no link
// against libcuda): the allocation an address lies in.
using PfnGetAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
static PfnGetAddressRange address_range_fn() {
  static PfnGetAddressRange fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnGetAddressRange>(p);
    cudaGetLastError();
  });
  return fn;
}

extern "C" walsh_status walsh_ipc_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  WALSH_CHECK_ARG(dev_ptr && handle_out && offset_out);
  auto range = address_range_fn();
  if (!range) return WALSH_ERR_NOT_INIT;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS) return WALSH_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, (void*)base) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)((CUdeviceptr)dev_ptr - base);
  return WALSH_OK;
}

extern "C" walsh_status walsh_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out, void** base_out) {
  WALSH_CHECK_ARG(handle && dev_ptr_out && base_out && offset >= 0);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  *base_out = p;
  *dev_ptr_out = (char*)p + offset;
  return WALSH_OK;
}

extern "C" walsh_status walsh_ipc_close(void* base) {
  WALSH_CHECK_ARG(base);
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return WALSH_ERR_LAUNCH;
  }
  return WALSH_OK;
}

extern "C" int walsh_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }
