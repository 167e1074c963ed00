// ThreadSanitizer driver for the host runtime (no torch, no Python):
// exercises the worker pool's job hand-off (thousands of short jobs,
// reconfiguration between jobs, jobs posted from two caller threads at once)
// and the AdamW range kernel run over the pool, then checks the results
// against a serial run.  Built and run by tests/test_host_tsan.py with
// -fsanitize=thread; any data race makes TSAN exit non-zero.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "../host_kernels.h"
#include "../thread_pool.h"

using t1h::AdamArgs;
using t1h::ThreadPool;

static void adam_over_pool(ThreadPool& pool, AdamArgs a, int64_t n, int64_t block) {
  const int64_t tasks = (n + block - 1) / block;
  pool.parallel_for(tasks, [&](int64_t t) {
    const int64_t b = t * block, e = std::min(n, b + block);
    t1h::adam_range_scalar(a, b, e);
  });
}

static AdamArgs make_args(std::vector<float>& p, std::vector<float>& g, std::vector<float>& m,
                          std::vector<float>& v) {
  AdamArgs a;
  std::memset(&a, 0, sizeof(a));
  a.param = p.data();
  a.param_dt = t1h::kF32;
  a.grad = g.data();
  a.grad_dt = t1h::kF32;
  a.exp_avg = m.data();
  a.exp_avg_sq = v.data();
  a.state_dt = t1h::kF32;
  a.h.beta1 = 0.9f;
  a.h.beta2 = 0.999f;
  a.h.one_minus_beta1 = 0.1f;
  a.h.one_minus_beta2 = 0.001f;
  a.h.eps = 1e-8f;
  a.h.bc2_rsqrt = 1.f / std::sqrt(1.f - 0.999f);
  a.h.step_size = -1e-3f / (1.f - 0.9f);
  a.h.wd = 0.01f;
  a.h.wd_step = -1e-3f * 0.01f;
  a.h.grad_scale = 1.f;
  a.h.adamw = 1;
  a.h.has_wd = 1;
  return a;
}

int main() {
  ThreadPool& pool = ThreadPool::instance();
  int failures = 0;

  // 1. many short jobs with reconfiguration in between
  for (int cfg : {4, 2, 6, 3}) {
    pool.configure(cfg, {});
    for (int it = 0; it < 2000; ++it) {
      std::atomic<int64_t> sum{0};
      pool.parallel_for(17, [&](int64_t t) { sum.fetch_add(t + 1, std::memory_order_relaxed); });
      if (sum.load() != 17 * 18 / 2) ++failures;
    }
  }

  // 2. two caller threads posting jobs concurrently (serialised by the pool)
  pool.configure(4, {});
  std::vector<int64_t> out_a(64, 0), out_b(64, 0);
  std::thread ta([&] {
    for (int it = 0; it < 500; ++it) pool.parallel_for(64, [&](int64_t t) { out_a[t] += 1; });
  });
  std::thread tb([&] {
    for (int it = 0; it < 500; ++it) pool.parallel_for(64, [&](int64_t t) { out_b[t] += 2; });
  });
  ta.join();
  tb.join();
  for (int i = 0; i < 64; ++i)
    if (out_a[i] != 500 || out_b[i] != 1000) ++failures;

  // 3. AdamW over the pool equals a serial run
  const int64_t n = 100003;
  std::vector<float> p(n), g(n), m(n, 0.f), v(n, 0.f);
  for (int64_t i = 0; i < n; ++i) {
    p[i] = std::sin(0.001f * i);
    g[i] = std::cos(0.003f * i);
  }
  std::vector<float> p2 = p, g2 = g, m2 = m, v2 = v;
  adam_over_pool(pool, make_args(p, g, m, v), n, 4096);
  t1h::adam_range_scalar(make_args(p2, g2, m2, v2), 0, n);
  for (int64_t i = 0; i < n; ++i)
    if (p[i] != p2[i] || m[i] != m2[i] || v[i] != v2[i]) {
      ++failures;
      break;
    }

  pool.configure(1, {});
  std::printf("race_driver: %s\n", failures ? "FAILED" : "ok");
  return failures ? 1 : 0;
}
