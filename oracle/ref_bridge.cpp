// Bridge that exposes the reference's own CPU kernels, compiled from the
// reference sources where they lie (src/b1_0_kernel.h, src/diffuser_types.h,
// included through -I), as plain C functions for the oracle and the CPU
// baseline.  It plays the role of ggml's CPU backend for these two custom
// ops: the callback is run once per worker with (ith, nth), exactly as
// ggml_backend_graph_compute does for a custom node (src/diffuser.cpp:269).
// Test infrastructure only: never linked into the product library.
#include "diffuser_types.h"
#include "b1_0_kernel.h"

#include <condition_variable>
#include <mutex>
#include <thread>
#include <vector>

namespace bonsai {
bool g_bonsai_debug = false;  // defined by the reference's drivers (src/diffuser.cpp:21-23)
}

namespace {
// A persistent worker pool, as ggml's CPU backend keeps one for the whole
// graph: the workers are created once and reused by every call, so a call's
// cost is the kernel's own work and not the creation of nth threads.  The
// calling thread runs ith = 0 itself; workers 1 .. nth-1 run the rest.
class Pool {
 public:
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      quit_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void run(ggml_custom_op_t fn, ggml_tensor* dst, int nth, void* ud) {
    if (nth <= 1) {
      fn(dst, 0, 1, ud);
      return;
    }
    std::lock_guard<std::mutex> call(call_mu_);  // one call at a time
    grow(nth - 1);
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = fn;
      dst_ = dst;
      ud_ = ud;
      nth_ = nth;
      pending_ = nth - 1;
      ++gen_;
    }
    cv_.notify_all();
    fn(dst, 0, nth, ud);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
  }

 private:
  // Called with call_mu_ held, before the call's generation is published: a
  // new worker starts from the current generation and so joins that call.
  void grow(int n) {
    while ((int)workers_.size() < n) {
      const int ith = (int)workers_.size() + 1;
      unsigned long long g0;
      {
        std::lock_guard<std::mutex> lk(mu_);
        g0 = gen_;
      }
      workers_.emplace_back([this, ith, g0] { loop(ith, g0); });
    }
  }
  void loop(int ith, unsigned long long seen) {
    for (;;) {
      ggml_custom_op_t fn;
      ggml_tensor* dst;
      void* ud;
      int nth;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (quit_) return;
        fn = fn_;
        dst = dst_;
        ud = ud_;
        nth = nth_;
      }
      if (ith >= nth) continue;
      fn(dst, ith, nth, ud);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  std::vector<std::thread> workers_;
  ggml_custom_op_t fn_ = nullptr;
  ggml_tensor* dst_ = nullptr;
  void* ud_ = nullptr;
  int nth_ = 0, pending_ = 0;
  unsigned long long gen_ = 0;
  bool quit_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

void run_threads(ggml_custom_op_t fn, ggml_tensor* dst, int nth, void* ud) {
  pool().run(fn, dst, nth, ud);
}
}  // namespace

extern "C" {

// out[t][r] for act f32 [tokens][in_dim], w = packed [out_dim][in_dim/32][6].
// Calls bonsai::b1_linear_f32_f32 (src/b1_0_kernel.h:37-288) with the tensor
// shapes b1_linear() builds (src/b1_0_kernel.h:290-300).
void ref_b1_linear(const float* act, int tokens, int in_dim, const uint8_t* w, int out_dim,
                   float* out, int nthreads) {
  ggml_tensor a{}, wt{}, dst{};
  a.type = GGML_TYPE_F32;
  a.ne[0] = in_dim; a.ne[1] = tokens; a.ne[2] = 1; a.ne[3] = 1;
  a.data = const_cast<float*>(act);
  wt.type = GGML_TYPE_I8;
  wt.ne[0] = (int64_t)out_dim * (in_dim / 32) * 6; wt.ne[1] = 1; wt.ne[2] = 1; wt.ne[3] = 1;
  wt.data = const_cast<uint8_t*>(w);
  dst.type = GGML_TYPE_F32;
  dst.ne[0] = out_dim; dst.ne[1] = tokens; dst.ne[2] = 1; dst.ne[3] = 1;
  dst.src[0] = &a;
  dst.src[1] = &wt;
  dst.data = out;
  bonsai::B1LinearUserData ud;
  ud.in_dim = in_dim;
  ud.out_dim = out_dim;
  run_threads(bonsai::b1_linear_f32_f32, &dst, nthreads, &ud);
}

// rope_2d_fwd_f32 (src/b1_0_kernel.h:309-361): x/out f32 [seq][n_heads][head_dim],
// cos/sin f32 [seq][head_dim/2].
void ref_rope_2d(const float* x, const float* c, const float* s, int head_dim, int n_heads,
                 int seq, float* out, int nthreads) {
  ggml_tensor xt{}, ct{}, st{}, dst{};
  xt.type = ct.type = st.type = dst.type = GGML_TYPE_F32;
  xt.data = const_cast<float*>(x);
  ct.data = const_cast<float*>(c);
  st.data = const_cast<float*>(s);
  dst.ne[0] = head_dim; dst.ne[1] = n_heads; dst.ne[2] = seq; dst.ne[3] = 1;
  dst.src[0] = &xt; dst.src[1] = &ct; dst.src[2] = &st;
  dst.data = out;
  bonsai::Rope2DUserData ud;
  ud.head_dim = head_dim;
  ud.n_heads = n_heads;
  ud.seq = seq;
  run_threads(bonsai::rope_2d_fwd_f32, &dst, nthreads, &ud);
}

int ref_has_avx2(void) {
#ifdef __AVX2__
  return 1;
#else
  return 0;
#endif
}
}
