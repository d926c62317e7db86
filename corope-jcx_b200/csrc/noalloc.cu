// corope_bwd_noalloc: the backward for callers that cannot allocate device
// memory.
//
// Some hosts own all device memory and give a plugin no way to allocate:
// an inference or training engine whose plugin interface hands over only
// input and output buffers (no workspace), or a runtime that runs under a
// fixed, pre-reserved memory budget where a cudaMalloc from inside a layer
// would fail or stall the whole process.  Such callers cannot provide the
// workspace corope_bwd asks for.  This entry point instead uses a scratch
// buffer that is part of the library image: a file-scope __device__ array of
// kScratchBytes (64 MiB), which every GPU that loads the library keeps until
// the process exits.  The caller still passes every input and output.
//
// Limits and rules:
//   * the backward's scratch (two fp32 rows [B,H,S], the tensor-core path's
//     128 KiB table of expansion coefficients, and fp32 dk/dv accumulators
//     [B,Hkv,S,D]) must fit in 64 MiB, otherwise the call returns
//     COROPE_ERR_WORKSPACE and does nothing;
//   * the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture;
//   * all calls on a device share the one array, and each call overwrites
//     it (the accumulator part is cleared on the call's stream before use),
//     so calls whose executions overlap on the GPU race -- serialise them
//     (one stream, or events between streams);
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace corope {
// corope_api.cu
int set_last_error(int code, const char* msg);
int bwd_check_args(const corope_bwd_params_t* p);
int device_check();
}

namespace {

constexpr size_t kScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_bwd_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" {

int corope_bwd(const corope_bwd_params_t* p, corope_stream_t stream);
size_t corope_bwd_min_workspace_bytes(const corope_bwd_params_t* p);

size_t corope_bwd_noalloc_scratch_bytes(void) { return kScratchBytes; }

int corope_bwd_noalloc(const corope_bwd_params_t* p, corope_stream_t stream) {
  // the same statuses, in the same order, as corope_bwd: arguments, then the
  // scratch size (in place of the workspace), then the device
  int rc = corope::bwd_check_args(p);
  if (rc) return rc;
  const size_t need = corope_bwd_min_workspace_bytes(p);
  if (need > kScratchBytes) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "corope_bwd_noalloc: this shape needs %zu bytes of scratch; the built-in scratch "
             "holds %zu bytes (use corope_bwd with a caller workspace)",
             need, kScratchBytes);
    return corope::set_last_error(COROPE_ERR_WORKSPACE, msg);
  }
  if ((rc = corope::device_check())) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return corope::set_last_error(COROPE_ERR_CUDA, "corope_bwd_noalloc: no usable current device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
      void* addr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress((void**)&addr, g_bwd_scratch);
      if (e != cudaSuccess || !addr)
        return corope::set_last_error(COROPE_ERR_CUDA,
                                      "corope_bwd_noalloc: cudaGetSymbolAddress of the scratch failed");
      g_scratch_ptr[dev] = addr;
    }
    scratch = g_scratch_ptr[dev];
  }
  corope_bwd_params_t q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kScratchBytes;  // what is left after the minimum may serve as hand-off
  return corope_bwd(&q, stream);
}

}  // extern "C"
