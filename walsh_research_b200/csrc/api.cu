// Library-wide entry points: status strings, ABI version, host-side fault
// injection and launch-status mapping.
#include <stdlib.h>
#include <string.h>

#include "common.cuh"

namespace walsh {

int injected(const char* site) {
  const char* v = getenv("WALSH_INJECT_FAULT");
  if (!v || !*v) return 0;
  if (strcmp(v, "all") == 0 || strcmp(v, site) == 0) return WALSH_ERR_INJECTED;
  return 0;
}

int launch_status() {
  const cudaError_t e = cudaPeekAtLastError();
  if (e == cudaSuccess) return WALSH_OK;
  cudaGetLastError();  // clear a sticky-free launch error so later calls are unaffected
  return WALSH_ERR_LAUNCH;
}

}  // namespace walsh

extern "C" const char* walsh_status_str(walsh_status s) {
  switch (s) {
    case WALSH_OK: return "ok";
    case WALSH_ERR_ARG: return "invalid argument (null pointer or bad scalar)";
    case WALSH_ERR_SHAPE: return "unsupported or inconsistent shape";
    case WALSH_ERR_DTYPE: return "unknown dtype code";
    case WALSH_ERR_ALIGN: return "pointer misaligned";
    case WALSH_ERR_LAUNCH: return "CUDA kernel launch failed";
    case WALSH_ERR_TIMEOUT: return "bounded device wait timed out";
    case WALSH_ERR_INJECTED: return "fault injected by WALSH_INJECT_FAULT";
    case WALSH_ERR_NOT_INIT: return "library not initialised for this device";
    case WALSH_ERR_INDEX: return "token id out of range";
    case WALSH_ERR_SCRATCH: return "problem needs more scratch than the fixed array of an allocation-free entry point";
    default: return "unknown walsh status";
  }
}

extern "C" int walsh_abi_version(void) { return 2; }
