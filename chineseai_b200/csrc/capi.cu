// capi.cu - status handling shared by every entry point of the cnnue library.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace cnnue {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_error(cudaError_t err, const char* what) {
  return set_error(CNNUE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(err),
                   cudaGetErrorName(err));
}

PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int status_from_word(uint32_t word) {
  int st = CNNUE_OK;
  if (word & CNNUE_STATUS_BAD_OFFSETS)
    st = CNNUE_ERR_BAD_OFFSETS;
  else if (word & CNNUE_STATUS_BAD_INDEX)
    st = CNNUE_ERR_BAD_INDEX;
  else if (word & CNNUE_STATUS_TIMEOUT)
    st = CNNUE_ERR_TIMEOUT;
  else if (word != 0)
    st = CNNUE_ERR_INTERNAL;
  if (st != CNNUE_OK) set_error(st, "kernel status word 0x%x", word);
  return st;
}

int use_device(int device) {
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (cur != device) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  }
  return CNNUE_OK;
}

}  // namespace cnnue

extern "C" {

const char* cnnue_status_string(int status) {
  switch (status) {
    case CNNUE_OK: return "ok";
    case CNNUE_ERR_INVALID_ARG: return "invalid argument";
    case CNNUE_ERR_BAD_INDEX: return "feature index out of range";
    case CNNUE_ERR_BAD_OFFSETS: return "offsets not monotone or beyond the index array";
    case CNNUE_ERR_CUDA: return "CUDA error";
    case CNNUE_ERR_WORKSPACE: return "workspace too small";
    case CNNUE_ERR_FORMAT: return "bad weight format";
    case CNNUE_ERR_IO: return "I/O error";
    case CNNUE_ERR_NO_DEVICE: return "no such CUDA device";
    case CNNUE_ERR_TIMEOUT: return "device-side wait timed out";
    case CNNUE_ERR_INTERNAL: return "kernel self-check failed";
    default: return "unknown status";
  }
}

const char* cnnue_last_error(void) { return cnnue::g_last_error; }

const char* cnnue_version(void) { return "0.1.0"; }

int cnnue_read_status(void* d_workspace, void* stream, int* status_out) {
  if (!d_workspace || !status_out)
    return cnnue::set_error(CNNUE_ERR_INVALID_ARG, "null workspace or status_out");
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t word = 0;
  CNNUE_CUDA_TRY(cudaMemcpyAsync(&word, d_workspace, 4, cudaMemcpyDeviceToHost, s));
  CNNUE_CUDA_TRY(cudaStreamSynchronize(s));
  CNNUE_CUDA_TRY(cudaMemsetAsync(d_workspace, 0, 4, s));
  *status_out = cnnue::status_from_word(word);
  return CNNUE_OK;
}

}  // extern "C"

namespace cnnue {

DeviceGuard::DeviceGuard(int device) {
  if (cudaGetDevice(&prev) != cudaSuccess) {
    status = set_error(CNNUE_ERR_NO_DEVICE, "cudaGetDevice failed");
    return;
  }
  if (prev != device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
      status = cuda_error(e, "cudaSetDevice");
      return;
    }
    switched = true;
  }
}

DeviceGuard::~DeviceGuard() {
  if (switched) cudaSetDevice(prev);
}

int check_launch_error(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  return CNNUE_OK;
}

}  // namespace cnnue
