// Runtime plumbing of the C ABI: error reporting, device error word,
// launch accounting, B1_0 weight upload and the op-level B1_0 entry points.
#include "../../include/bonsai_cuda.h"
#include "internal.cuh"
#include "ptx.cuh"

#include <cuda_fp16.h>
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace bonsai {

namespace {
thread_local std::string g_last_error;
thread_local long long g_launches = 0;

// Per-device error word written by kernels whose bounded waits expire.
__device__ int g_device_error_word;

struct DeviceInfo {
  int* err_word = nullptr;
  int sms = 0;
  bool checked = false;
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

DeviceInfo& dev_info() {
  int d = 0;
  cudaGetDevice(&d);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& di = g_dev[d & 63];
  if (!di.checked) {
    di.checked = true;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) == cudaSuccess)
      di.err_word = static_cast<int*>(p);
    cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d);
    if (di.sms <= 0) di.sms = 148;
  }
  return di;
}

// Scratch f16 copy of the f32 activations used by bonsai_b1_linear_f32, one
// per (device, stream) of the calling thread: calls on different streams
// never share a buffer, so one stream's call cannot overwrite the copy that
// another stream's GEMM is still reading, and a buffer is grown or freed only
// in the order of its own stream.  `done` is recorded after every use and
// waited on by the next one, which keeps a buffer safe even when a destroyed
// stream's handle is reused by a new stream while the old work still runs.
struct Scratch {
  int device = -1;
  cudaStream_t stream = nullptr;
  void* ptr = nullptr;
  size_t bytes = 0;
  cudaEvent_t done = nullptr;
};
thread_local std::vector<Scratch> g_scratch;

Scratch* scratch_for(int device, cudaStream_t st) {
  for (auto& s : g_scratch)
    if (s.device == device && s.stream == st) return &s;
  Scratch s;
  s.device = device;
  s.stream = st;
  if (cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  g_scratch.push_back(s);
  return &g_scratch.back();
}

__global__ void f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst,
                                  long long n) {
  long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4;
  const long long stride = (long long)gridDim.x * blockDim.x * 4;
  for (; i < n; i += stride) {
    if (i + 3 < n) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      __half2 a = __floats2half2_rn(v.x, v.y);
      __half2 b = __floats2half2_rn(v.z, v.w);
      *reinterpret_cast<__half2*>(dst + i) = a;
      *reinterpret_cast<__half2*>(dst + i + 2) = b;
    } else {
      for (long long j = i; j < n; ++j) dst[j] = __float2half_rn(src[j]);
    }
  }
}
__global__ void f32_to_f16_scalar_kernel(const float* __restrict__ src, __half* __restrict__ dst,
                                         long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}
}  // namespace

int device_slot() {
  int d = 0;
  cudaGetDevice(&d);
  return d & 63;
}

void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 0;
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return BONSAI_ERR_CUDA;
}
int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    ++g_launches;
    return 0;
  }
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return BONSAI_ERR_CUDA;
}
// ------------------------------------------------------------ profiling
// When enabled, each launch site brackets its kernel with two CUDA events
// recorded on the launching stream and logs the algorithmic work of the
// launch; bonsai_profile_stop() turns that into per-kernel totals.
namespace {
struct ProfRec {
  const char* kind;
  cudaEvent_t e0, e1;
  double flop, bytes;
};
thread_local bool g_prof_on = false;
thread_local std::vector<ProfRec> g_prof;
}  // namespace

ProfScope::ProfScope(const char* kind, double flop, double bytes, cudaStream_t st) : st_(st) {
  if (!g_prof_on) return;
  ProfRec r{kind, nullptr, nullptr, flop, bytes};
  if (cudaEventCreate(&r.e0) != cudaSuccess || cudaEventCreate(&r.e1) != cudaSuccess) return;
  cudaEventRecord(r.e0, st);
  g_prof.push_back(r);
  idx_ = (long long)g_prof.size() - 1;
}
ProfScope::~ProfScope() {
  if (idx_ >= 0 && idx_ < (long long)g_prof.size()) cudaEventRecord(g_prof[idx_].e1, st_);
}

int* device_error_word() { return dev_info().err_word; }
long long launch_counter() { return g_launches; }
void launch_counter_add(long long n) { g_launches += n; }
bool profiling_active() { return g_prof_on; }
int num_sms() { return dev_info().sms; }

int launch_f32_to_f16(const float* src, __half* dst, long long n, cudaStream_t st) {
  if (n <= 0) return 0;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(src) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(dst) & 7) == 0);
  const int threads = 256;
  long long blocks = (n / 4 + threads - 1) / threads;
  blocks = std::max<long long>(1, std::min<long long>(blocks, (long long)num_sms() * 8));
  if (vec_ok)
    f32_to_f16_kernel<<<(unsigned)blocks, threads, 0, st>>>(src, dst, n);
  else
    f32_to_f16_scalar_kernel<<<(unsigned)blocks, threads, 0, st>>>(src, dst, n);
  return launch_status("f32_to_f16 launch");
}

}  // namespace bonsai

using namespace bonsai;

#define RC_CUDA(call, what)                                \
  do {                                                     \
    const cudaError_t _e = (call);                         \
    if (_e != cudaSuccess) return cuda_status(_e, (what)); \
  } while (0)

extern "C" {

const char* bonsai_last_error(void) { return g_last_error.c_str(); }

long long bonsai_launch_count(void) {
  long long n = g_launches;
  g_launches = 0;
  return n;
}

int bonsai_init(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(BONSAI_ERR_UNSUPPORTED,
                "bonsai_init: device " + std::to_string(device) + " is sm_" +
                    std::to_string(prop.major) + std::to_string(prop.minor) +
                    "; this library is built for sm_100a only");
  dev_info();
  g_last_error.clear();
  return 0;
}

int bonsai_shutdown(void) {
  // Waits for the device, then releases what the library allocated lazily for
  // this host thread on the current device (the f16 activation scratch of
  // bonsai_b1_linear_f32) and any pending profiling events.  Weight handles
  // and models stay valid until their own free/destroy calls.
  int d = 0;
  cudaGetDevice(&d);
  const cudaError_t e = cudaDeviceSynchronize();
  for (size_t i = 0; i < g_scratch.size();) {
    Scratch& sc = g_scratch[i];
    if (sc.device != d) {
      ++i;
      continue;
    }
    if (sc.ptr) cudaFree(sc.ptr);
    if (sc.done) cudaEventDestroy(sc.done);
    g_scratch.erase(g_scratch.begin() + i);
  }
  for (auto& r : g_prof) {
    cudaEventDestroy(r.e0);
    cudaEventDestroy(r.e1);
  }
  g_prof.clear();
  g_prof_on = false;
  return cuda_status(e, "bonsai_shutdown: device synchronize");
}

int bonsai_profile_start(void) {
  for (auto& r : g_prof) {
    cudaEventDestroy(r.e0);
    cudaEventDestroy(r.e1);
  }
  g_prof.clear();
  g_prof_on = true;
  return 0;
}

int bonsai_profile_stop(char* json, int cap) {
  g_prof_on = false;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "profile sync");
  struct Acc {
    long long n = 0;
    double ms = 0, flop = 0, bytes = 0;
  };
  std::vector<std::pair<std::string, Acc>> acc;
  for (auto& r : g_prof) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.e0, r.e1);
    auto it = std::find_if(acc.begin(), acc.end(), [&](auto& a) { return a.first == r.kind; });
    if (it == acc.end()) {
      acc.push_back({r.kind, Acc{}});
      it = acc.end() - 1;
    }
    it->second.n += 1;
    it->second.ms += ms;
    it->second.flop += r.flop;
    it->second.bytes += r.bytes;
    cudaEventDestroy(r.e0);
    cudaEventDestroy(r.e1);
  }
  g_prof.clear();
  std::string out = "{";
  for (size_t i = 0; i < acc.size(); ++i) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s\"%s\": {\"launches\": %lld, \"ms\": %.6f, \"flop\": %.6e, \"bytes\": %.6e}",
             i ? ", " : "", acc[i].first.c_str(), acc[i].second.n, acc[i].second.ms,
             acc[i].second.flop, acc[i].second.bytes);
    out += buf;
  }
  out += "}";
  if (json && cap > 0) {
    const size_t n = std::min<size_t>(out.size(), (size_t)cap - 1);
    memcpy(json, out.data(), n);
    json[n] = 0;
  }
  return (int)out.size();
}

int bonsai_device_error(void) {
  int* w = device_error_word();
  if (!w) return fail(BONSAI_ERR_CUDA, "device error word unavailable");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "read device error word");
  if (v != 0) {
    int z = 0;
    cudaMemcpy(w, &z, sizeof(int), cudaMemcpyHostToDevice);
  }
  return v;
}

int bonsai_b1_upload(const uint8_t* host_packed, int out_dim, int in_dim, int swiglu_from,
                     bonsai_b1_t* out) {
  if (!out) return fail(BONSAI_ERR_ARG, "b1_upload: null output handle");
  *out = nullptr;
  if (!host_packed || out_dim <= 0 || in_dim <= 0)
    return fail(BONSAI_ERR_ARG, "b1_upload: null data or non-positive shape");
  if (in_dim % BONSAI_B1_BLOCK_SIZE != 0)
    return fail(BONSAI_ERR_ARG, "b1_upload: in_dim must be a multiple of 32");
  if (swiglu_from >= 0) {
    if (swiglu_from >= out_dim || ((out_dim - swiglu_from) & 1) || (swiglu_from & 1))
      return fail(BONSAI_ERR_ARG,
                  "b1_upload: swiglu_from must be even and leave an even number of rows");
  }
  auto* h = new bonsai_b1_weight();
  B1Weight& w = h->w;
  w.n_rows = out_dim;
  w.k_in = in_dim;
  w.n_ftiles = (out_dim + 127) / 128;
  w.k_blocks = (in_dim + 63) / 64;
  w.swiglu_from = swiglu_from;
  cudaGetDevice(&w.device);
  const size_t packed = (size_t)out_dim * (in_dim / 32) * 6;
  const size_t chunk_bytes = (size_t)w.n_ftiles * w.k_blocks * kChunkWords * 4;
  uint8_t* tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, packed);
  if (e != cudaSuccess) {
    delete h;
    return fail(BONSAI_ERR_NOMEM, "b1_upload: cudaMalloc staging failed");
  }
  e = cudaMalloc(&w.chunks, chunk_bytes);
  if (e != cudaSuccess) {
    cudaFree(tmp);
    delete h;
    return fail(BONSAI_ERR_NOMEM, "b1_upload: cudaMalloc weights failed");
  }
  e = cudaMemcpy(tmp, host_packed, packed, cudaMemcpyHostToDevice);
  int rc = (e == cudaSuccess) ? launch_b1_retile(tmp, w, 0) : cuda_status(e, "b1_upload copy");
  if (rc == 0) rc = cuda_status(cudaDeviceSynchronize(), "b1_upload retile");
  cudaFree(tmp);
  if (rc) {
    cudaFree(w.chunks);
    delete h;
    return rc;
  }
  *out = h;
  return 0;
}

int bonsai_b1_free(bonsai_b1_t h) {
  if (!h) return 0;
  cudaFree(h->w.chunks);
  delete h;
  return 0;
}

int bonsai_b1_shape(bonsai_b1_t h, int* out_dim, int* in_dim) {
  if (!h) return fail(BONSAI_ERR_ARG, "b1_shape: null handle");
  if (out_dim) *out_dim = h->w.n_rows;
  if (in_dim) *in_dim = h->w.k_in;
  return 0;
}

int bonsai_b1_gemm(const uint16_t* x, long long ldx, int tokens, bonsai_b1_t h, int mode,
                   void* out, long long ld_out, const float* gate, void* stream) {
  if (!h) return fail(BONSAI_ERR_ARG, "b1_gemm: null weight handle");
  if (tokens == 0) return 0;
  if (!out) return fail(BONSAI_ERR_ARG, "b1_gemm: null output");
  const B1Weight& w = h->w;
  int dev = 0;
  RC_CUDA(cudaGetDevice(&dev), "b1_gemm: cudaGetDevice");
  if (dev != w.device)
    return fail(BONSAI_ERR_ARG, "b1_gemm: the weight lives on device " + std::to_string(w.device) +
                                    ", the current device is " + std::to_string(dev));
  EpiSeg seg;
  seg.row_begin = 0;
  seg.row_end = w.n_rows;
  seg.dst = out;
  seg.ld = ld_out;
  seg.gate = gate;
  switch (mode) {
    case BONSAI_EPI_F32: seg.mode = EPI_F32; break;
    case BONSAI_EPI_F16: seg.mode = EPI_F16; break;
    case BONSAI_EPI_GELU: seg.mode = EPI_GELU_F16; break;
    case BONSAI_EPI_RESID: seg.mode = EPI_RESID_F32; break;
    case BONSAI_EPI_SWIGLU:
      if (w.swiglu_from != 0)
        return fail(BONSAI_ERR_ARG, "b1_gemm: SWIGLU needs a weight uploaded with swiglu_from=0");
      seg.mode = EPI_SWIGLU_F16;
      break;
    default: return fail(BONSAI_ERR_ARG, "b1_gemm: unknown epilogue mode");
  }
  const long long need = (mode == BONSAI_EPI_SWIGLU) ? w.n_rows / 2 : w.n_rows;
  if (ld_out < need) return fail(BONSAI_ERR_ARG, "b1_gemm: ld_out smaller than the output width");
  return launch_b1_gemm(x, ldx, tokens, w, &seg, 1, false, static_cast<cudaStream_t>(stream));
}

int bonsai_b1_linear_f32(const float* act, int tokens, bonsai_b1_t h, float* out, void* stream) {
  if (!h) return fail(BONSAI_ERR_ARG, "b1_linear_f32: null weight handle");
  if (tokens < 0) return fail(BONSAI_ERR_ARG, "b1_linear_f32: negative token count");
  if (tokens == 0) return 0;  // empty batch: nothing to do (pointers may be null)
  if (!act || !out) return fail(BONSAI_ERR_ARG, "b1_linear_f32: null tensor");
  const B1Weight& w = h->w;
  int dev = 0;
  RC_CUDA(cudaGetDevice(&dev), "b1_linear_f32: cudaGetDevice");
  if (dev != w.device)
    return fail(BONSAI_ERR_ARG, "b1_linear_f32: the weight lives on device " +
                                    std::to_string(w.device) + ", the current device is " +
                                    std::to_string(dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // One token: the memory-bound matrix-vector kernel on the f32 activations
  // (a tensor-core tile would be almost all padding); no scratch.
  if (tokens == 1 && b1_gemv_supported(w)) return launch_b1_gemv_f32(act, w, out, st);
  // f16 copy of the activations; K is padded to a multiple of 8 so that
  // the TMA row pitch is 16-byte aligned (K % 32 == 0 already guarantees it).
  const long long n = (long long)tokens * w.k_in;
  Scratch* sc = scratch_for(dev, st);
  if (!sc) return fail(BONSAI_ERR_CUDA, "b1_linear_f32: scratch event creation failed");
  // the previous use of this buffer (in this stream's order, or of a stream
  // that had the same handle) has finished before it is overwritten or freed
  RC_CUDA(cudaStreamWaitEvent(st, sc->done, 0), "b1_linear_f32: wait for the scratch");
  const size_t need = (size_t)n * sizeof(__half);
  if (sc->bytes < need) {
    if (sc->ptr) cudaFreeAsync(sc->ptr, st);
    sc->ptr = nullptr;
    sc->bytes = 0;
    cudaError_t e = cudaMallocAsync(&sc->ptr, need, st);
    if (e != cudaSuccess) return fail(BONSAI_ERR_NOMEM, "b1_linear_f32: scratch allocation failed");
    sc->bytes = need;
  }
  int rc = launch_f32_to_f16(act, static_cast<__half*>(sc->ptr), n, st);
  if (rc) return rc;
  EpiSeg seg;
  seg.mode = EPI_F32;
  seg.row_begin = 0;
  seg.row_end = w.n_rows;
  seg.dst = out;
  seg.ld = w.n_rows;
  rc = launch_b1_gemm(sc->ptr, w.k_in, tokens, w, &seg, 1, false, st);
  if (rc) return rc;
  return cuda_status(cudaEventRecord(sc->done, st), "b1_linear_f32: record the scratch's use");
}

}  // extern "C"
