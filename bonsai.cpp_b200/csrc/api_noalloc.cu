// bonsai_b1_linear_f32_noalloc: the drop-in B1_0 linear for callers that
// must not have the library allocate device memory.
//
// bonsai_b1_linear_f32 keeps an f16 copy of the activations in a scratch
// buffer that it grows with cudaMallocAsync.  Some hosts cannot allow that:
// a ggml-style backend whose graph allocator owns every device byte, or a
// latency-critical loop where an allocation (and the synchronisation it may
// cause) is not acceptable.
// This entry point instead uses one fixed array that lives in the library's
// device image: kNoAllocMaxElems f16 values (8 MiB), which every GPU that
// loads the library keeps reserved until the process exits.
#include "../../include/bonsai_cuda.h"
#include "internal.cuh"

#include <mutex>

namespace bonsai {
namespace {

constexpr long long kNoAllocMaxElems = 4LL << 20;  // tokens * in_dim <= 4,194,304 (8 MiB of f16)

// The scratch array.  In host code this symbol is only a stand-in: its
// device address comes from cudaGetSymbolAddress below, once per device.
static __device__ __align__(256) __half g_noalloc_scratch[kNoAllocMaxElems];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device (resolved on
// the first call made on that device, with that device current).
int noalloc_scratch(__half** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "b1_linear_f32_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(BONSAI_ERR_UNSUPPORTED, "b1_linear_f32_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return cuda_status(e, "b1_linear_f32_noalloc: cudaGetSymbolAddress of the scratch array");
    g_noalloc_ptr[dev] = p;
  }
  *out = static_cast<__half*>(g_noalloc_ptr[dev]);
  return 0;
}

}  // namespace
}  // namespace bonsai

using namespace bonsai;

extern "C" int bonsai_b1_linear_f32_noalloc(const float* act, int tokens, bonsai_b1_t h,
                                            float* out, void* stream) {
  if (!h) return fail(BONSAI_ERR_ARG, "b1_linear_f32_noalloc: null weight handle");
  if (tokens < 0) return fail(BONSAI_ERR_ARG, "b1_linear_f32_noalloc: negative token count");
  if (tokens == 0) return 0;
  if (!act || !out) return fail(BONSAI_ERR_ARG, "b1_linear_f32_noalloc: null tensor");
  const B1Weight& w = h->w;
  int cur = 0;
  cudaError_t ce = cudaGetDevice(&cur);
  if (ce != cudaSuccess) return cuda_status(ce, "b1_linear_f32_noalloc: cudaGetDevice");
  // One token: the same f32 matrix-vector kernel as bonsai_b1_linear_f32
  // (it needs no activation copy, so neither the scratch array nor a size limit).
  if (tokens == 1 && b1_gemv_supported(w)) {
    if (cur != w.device)
      return fail(BONSAI_ERR_ARG, "b1_linear_f32_noalloc: the weight lives on device " +
                                      std::to_string(w.device) + ", the current device is " +
                                      std::to_string(cur));
    return launch_b1_gemv_f32(act, w, out, static_cast<cudaStream_t>(stream));
  }
  const long long n = (long long)tokens * w.k_in;
  if (n > kNoAllocMaxElems)
    return fail(BONSAI_ERR_UNSUPPORTED,
                "b1_linear_f32_noalloc: tokens * in_dim = " + std::to_string(n) +
                    " exceeds the fixed scratch of " + std::to_string(kNoAllocMaxElems) +
                    " elements (8 MiB); split the call or use bonsai_b1_linear_f32");
  __half* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != w.device)
    return fail(BONSAI_ERR_ARG, "b1_linear_f32_noalloc: the weight lives on device " +
                                    std::to_string(w.device) + ", the current device is " +
                                    std::to_string(dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every element the GEMM reads (tokens x in_dim) is written here first, so
  // nothing is left over from an earlier call's contents.
  rc = launch_f32_to_f16(act, scratch, n, st);
  if (rc) return rc;
  EpiSeg seg;
  seg.mode = EPI_F32;
  seg.row_begin = 0;
  seg.row_end = w.n_rows;
  seg.dst = out;
  seg.ld = w.n_rows;
  return launch_b1_gemm(scratch, w.k_in, tokens, w, &seg, 1, false, st);
}
