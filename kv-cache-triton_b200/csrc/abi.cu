// Status strings and CUDA-error bookkeeping of the C ABI.
#include <string.h>

#include "common.cuh"

namespace kv4 {

static thread_local char g_last_cuda[256] = "";

void set_cuda_error(cudaError_t e) {
  const char *s = cudaGetErrorString(e);
  strncpy(g_last_cuda, s ? s : "unknown CUDA error", sizeof(g_last_cuda) - 1);
  g_last_cuda[sizeof(g_last_cuda) - 1] = 0;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return KV4_OK;
  set_cuda_error(e);
  return KV4_ERR_CUDA;
}

}  // namespace kv4

extern "C" int kv4_version(void) { return 100; }

extern "C" const char *kv4_last_cuda_error(void) { return kv4::g_last_cuda; }

extern "C" const char *kv4_strerror(int status) {
  switch (status) {
    case KV4_OK: return "ok";
    case KV4_ERR_INVALID: return "invalid argument";
    case KV4_ERR_DTYPE: return "unsupported dtype";
    case KV4_ERR_SHAPE: return "inconsistent shapes";
    case KV4_ERR_LAYOUT: return "unsupported strides or alignment";
    case KV4_ERR_WORKSPACE: return "workspace missing or too small";
    case KV4_ERR_CUDA: return "CUDA runtime error";
    case KV4_ERR_UNSUPPORTED: return "unsupported configuration";
    case KV4_ERR_DEVICE: return "device-side error (bounded wait expired)";
    case KV4_ERR_SCRATCH_LIMIT:
      return "request needs more scratch than kv4_attention_noalloc's fixed 4 MiB area";
    default: return "unknown status";
  }
}
