// Host-side operations exposed to Python: ISA dispatch, threaded LayerAdam
// step, casts, slot reductions, shared-memory regions with bounded-wait
// counters, and NUMA placement.  All entry points that touch large buffers
// release the GIL.
#include <errno.h>
#include <fcntl.h>
#include <linux/mempolicy.h>
#include <sched.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <torch/extension.h>

#include "host_kernels.h"
#include "thread_pool.h"

namespace t1h {

// ------------------------------------------------------------- ISA dispatch
enum class Isa { kScalar = 0, kAvx2 = 1, kAvx512 = 2 };

static Isa detect_isa() {
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
      __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("fma"))
    return Isa::kAvx512;
  if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return Isa::kAvx2;
  return Isa::kScalar;
}

static Isa g_isa = detect_isa();

static const char* isa_name(Isa i) {
  switch (i) {
    case Isa::kAvx512: return "avx512";
    case Isa::kAvx2: return "avx2";
    default: return "scalar";
  }
}

std::string simd_level() { return isa_name(g_isa); }

// Force a narrower ISA (tests use this to exercise every variant).
void set_simd_level(const std::string& name) {
  Isa best = detect_isa();
  Isa want = name == "avx512" ? Isa::kAvx512 : name == "avx2" ? Isa::kAvx2 : Isa::kScalar;
  TORCH_CHECK(static_cast<int>(want) <= static_cast<int>(best), "CPU does not support ", name);
  g_isa = want;
}

static void adam_range(const AdamArgs& a, int64_t b, int64_t e) {
  switch (g_isa) {
    case Isa::kAvx512: return adam_range_avx512(a, b, e);
    case Isa::kAvx2: return adam_range_avx2(a, b, e);
    default: return adam_range_scalar(a, b, e);
  }
}
static void cast_range(const void* s, int sdt, void* d, int ddt, float sc, int64_t b, int64_t e) {
  switch (g_isa) {
    case Isa::kAvx512: return cast_range_avx512(s, sdt, d, ddt, sc, b, e);
    case Isa::kAvx2: return cast_range_avx2(s, sdt, d, ddt, sc, b, e);
    default: return cast_range_scalar(s, sdt, d, ddt, sc, b, e);
  }
}
static void sum_slots_range(const void* const* s, int n, int sdt, void* d, int ddt, float sc,
                            int64_t b, int64_t e) {
  switch (g_isa) {
    case Isa::kAvx512: return sum_slots_range_avx512(s, n, sdt, d, ddt, sc, b, e);
    case Isa::kAvx2: return sum_slots_range_avx2(s, n, sdt, d, ddt, sc, b, e);
    default: return sum_slots_range_scalar(s, n, sdt, d, ddt, sc, b, e);
  }
}
static void split_range(const float* s, uint16_t* hi, uint16_t* lo, int64_t b, int64_t e) {
  switch (g_isa) {
    case Isa::kAvx512: return split_range_avx512(s, hi, lo, b, e);
    case Isa::kAvx2: return split_range_avx2(s, hi, lo, b, e);
    default: return split_range_scalar(s, hi, lo, b, e);
  }
}
static void unsplit_range(const uint16_t* hi, const uint16_t* lo, float* d, int64_t b, int64_t e) {
  switch (g_isa) {
    case Isa::kAvx512: return unsplit_range_avx512(hi, lo, d, b, e);
    case Isa::kAvx2: return unsplit_range_avx2(hi, lo, d, b, e);
    default: return unsplit_range_scalar(hi, lo, d, b, e);
  }
}
static double sumsq_range(const void* s, int dt, int64_t b, int64_t e) {
  switch (g_isa) {
    case Isa::kAvx512: return sumsq_range_avx512(s, dt, b, e);
    case Isa::kAvx2: return sumsq_range_avx2(s, dt, b, e);
    default: return sumsq_range_scalar(s, dt, b, e);
  }
}

// ------------------------------------------------------------ threading
static constexpr int64_t kChunk = 1 << 16;  // elements per task (multiple of 64)

void configure_threads(int n, std::vector<int> cpus) {
  ThreadPool::instance().configure(n < 1 ? 1 : n, cpus);
}
int num_threads() { return ThreadPool::instance().num_threads(); }

template <class F>
static void chunked(int64_t n, F&& f) {
  int64_t tasks = (n + kChunk - 1) / kChunk;
  ThreadPool::instance().parallel_for(tasks, [&](int64_t t) {
    int64_t b = t * kChunk;
    int64_t e = b + kChunk < n ? b + kChunk : n;
    f(b, e);
  });
}

static int host_dt(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat32: return kF32;
    case torch::kBFloat16: return kBF16;
    case torch::kFloat16: return kF16;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return kF32;
}

static void check_cpu_contig(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.device().is_cpu(), what, " must be a CPU tensor");
  TORCH_CHECK(t.is_contiguous(), what, " must be contiguous (an update into a temporary copy "
              "would be lost)");
}

// ------------------------------------------------------------------ adam
AdamHyper make_hyper(int64_t step, double lr, double beta1, double beta2, double eps,
                     double wd, bool bias_correction, bool adamw, double grad_scale) {
  TORCH_CHECK(step >= 1, "Adam step counter must start at 1, got ", step);
  AdamHyper h;
  h.beta1 = static_cast<float>(beta1);
  h.beta2 = static_cast<float>(beta2);
  h.one_minus_beta1 = static_cast<float>(1.0 - beta1);
  h.one_minus_beta2 = static_cast<float>(1.0 - beta2);
  h.eps = static_cast<float>(eps);
  double bc1 = 1.0, bc2r = 1.0;
  if (bias_correction) {
    bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
    bc2r = 1.0 / std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step)));
  }
  h.bc2_rsqrt = static_cast<float>(bc2r);
  h.step_size = static_cast<float>(-lr / bc1);
  h.wd = static_cast<float>(wd);
  h.wd_step = static_cast<float>(-lr * wd);
  h.grad_scale = static_cast<float>(grad_scale);
  h.adamw = adamw ? 1 : 0;
  h.has_wd = wd > 0 ? 1 : 0;
  static const int stream_shadow = [] {
    const char* e = std::getenv("T1_STREAM_SHADOW");
    return (e != nullptr && e[0] == '0') ? 0 : 1;
  }();
  h.stream_shadow = stream_shadow;
  return h;
}

void adam_step(torch::Tensor param, c10::optional<torch::Tensor> grad, torch::Tensor exp_avg,
               torch::Tensor exp_avg_sq, c10::optional<torch::Tensor> shadow, int64_t step,
               double lr, double beta1, double beta2, double eps, double weight_decay,
               bool bias_correction, bool adamw_mode, double grad_scale) {
  check_cpu_contig(param, "param");
  check_cpu_contig(exp_avg, "exp_avg");
  check_cpu_contig(exp_avg_sq, "exp_avg_sq");
  const int64_t n = param.numel();
  TORCH_CHECK(exp_avg.numel() == n && exp_avg_sq.numel() == n, "state size mismatch");
  TORCH_CHECK(exp_avg.scalar_type() == exp_avg_sq.scalar_type(), "state dtypes differ");
  AdamArgs a;
  a.param = param.data_ptr();
  a.param_lo = nullptr;
  a.param_dt = host_dt(param);
  a.grad = nullptr;
  a.grad_dt = kF32;
  if (grad.has_value() && grad->defined()) {
    check_cpu_contig(*grad, "grad");
    TORCH_CHECK(grad->numel() == n, "grad size ", grad->numel(), " != param size ", n);
    a.grad = grad->data_ptr();
    a.grad_dt = host_dt(*grad);
  }
  a.exp_avg = exp_avg.data_ptr();
  a.exp_avg_sq = exp_avg_sq.data_ptr();
  a.state_dt = host_dt(exp_avg);
  a.shadow = nullptr;
  a.shadow_dt = kBF16;
  if (shadow.has_value() && shadow->defined()) {
    check_cpu_contig(*shadow, "shadow");
    TORCH_CHECK(shadow->numel() == n, "shadow size mismatch");
    a.shadow = shadow->data_ptr();
    a.shadow_dt = host_dt(*shadow);
  }
  a.h = make_hyper(step, lr, beta1, beta2, eps, weight_decay, bias_correction, adamw_mode,
                   grad_scale);
  pybind11::gil_scoped_release nogil;
  chunked(n, [&](int64_t b, int64_t e) { adam_range(a, b, e); });
}

// Adam on a split-plane master (hi plane = the bf16 copy, lo plane = the
// rest of the fp32 bits); no separate shadow is written.
void adam_step_split(torch::Tensor hi, torch::Tensor lo, c10::optional<torch::Tensor> grad,
                     torch::Tensor exp_avg, torch::Tensor exp_avg_sq, int64_t step, double lr,
                     double beta1, double beta2, double eps, double weight_decay,
                     bool bias_correction, bool adamw_mode, double grad_scale) {
  check_cpu_contig(hi, "hi");
  check_cpu_contig(lo, "lo");
  check_cpu_contig(exp_avg, "exp_avg");
  check_cpu_contig(exp_avg_sq, "exp_avg_sq");
  TORCH_CHECK(hi.element_size() == 2 && lo.element_size() == 2, "planes must be 16-bit");
  const int64_t n = hi.numel();
  TORCH_CHECK(lo.numel() == n && exp_avg.numel() == n && exp_avg_sq.numel() == n, "size mismatch");
  AdamArgs a;
  a.param = hi.data_ptr();
  a.param_lo = lo.data_ptr();
  a.param_dt = kSplit;
  a.grad = nullptr;
  a.grad_dt = kF32;
  if (grad.has_value() && grad->defined()) {
    check_cpu_contig(*grad, "grad");
    TORCH_CHECK(grad->numel() == n, "grad size mismatch");
    a.grad = grad->data_ptr();
    a.grad_dt = host_dt(*grad);
  }
  a.exp_avg = exp_avg.data_ptr();
  a.exp_avg_sq = exp_avg_sq.data_ptr();
  a.state_dt = host_dt(exp_avg);
  a.shadow = nullptr;
  a.shadow_dt = kBF16;
  a.h = make_hyper(step, lr, beta1, beta2, eps, weight_decay, bias_correction, adamw_mode,
                   grad_scale);
  pybind11::gil_scoped_release nogil;
  chunked(n, [&](int64_t b, int64_t e) { adam_range(a, b, e); });
}

// fp32 <-> split planes
void f32_to_split(torch::Tensor src, torch::Tensor hi, torch::Tensor lo) {
  check_cpu_contig(src, "src");
  check_cpu_contig(hi, "hi");
  check_cpu_contig(lo, "lo");
  TORCH_CHECK(src.scalar_type() == torch::kFloat32, "src must be fp32");
  const int64_t n = src.numel();
  TORCH_CHECK(hi.numel() == n && lo.numel() == n, "size mismatch");
  const float* s = src.data_ptr<float>();
  uint16_t* h = static_cast<uint16_t*>(hi.data_ptr());
  uint16_t* l = static_cast<uint16_t*>(lo.data_ptr());
  pybind11::gil_scoped_release nogil;
  chunked(n, [&](int64_t b, int64_t e) { split_range(s, h, l, b, e); });
}

void split_to_f32(torch::Tensor hi, torch::Tensor lo, torch::Tensor dst) {
  check_cpu_contig(dst, "dst");
  check_cpu_contig(hi, "hi");
  check_cpu_contig(lo, "lo");
  TORCH_CHECK(dst.scalar_type() == torch::kFloat32, "dst must be fp32");
  const int64_t n = dst.numel();
  TORCH_CHECK(hi.numel() == n && lo.numel() == n, "size mismatch");
  const uint16_t* h = static_cast<const uint16_t*>(hi.data_ptr());
  const uint16_t* l = static_cast<const uint16_t*>(lo.data_ptr());
  float* d = dst.data_ptr<float>();
  pybind11::gil_scoped_release nogil;
  chunked(n, [&](int64_t b, int64_t e) { unsplit_range(h, l, d, b, e); });
}

// ------------------------------------------------ reference-compatible API
// Mirrors the reference's cpu_adam module (create_adam / adam_update /
// destroy_adam, optimizer/layer_adam/csrc/cpu_adam.cpp:8-12) on top of
// adam_step.  Grads may be bf16/fp16 directly (no fp32 upcast needed).
struct AdamInstance {
  double lr, beta1, beta2, eps, wd;
  bool adamw;
};
static std::mutex g_inst_mu;
static std::unordered_map<int, AdamInstance> g_instances;

int create_adam(int id, double lr, double beta1, double beta2, double eps, double wd, bool adamw,
                bool should_log) {
  std::lock_guard<std::mutex> lk(g_inst_mu);
  g_instances[id] = AdamInstance{lr, beta1, beta2, eps, wd, adamw};
  if (should_log) {
    printf("LayerAdam host optimizer #%d created: simd=%s threads=%d adamw=%d\n", id,
           isa_name(g_isa), num_threads(), adamw ? 1 : 0);
  }
  return 0;
}

int adam_update(int id, int64_t step, double lr, double beta1, double beta2, double eps,
                double wd, bool bias_correction, torch::Tensor p, torch::Tensor g,
                torch::Tensor m, torch::Tensor v) {
  AdamInstance inst;
  {
    std::lock_guard<std::mutex> lk(g_inst_mu);
    auto it = g_instances.find(id);
    TORCH_CHECK(it != g_instances.end(), "no LayerAdam optimizer with id ", id);
    inst = it->second;
  }
  adam_step(p, g, m, v, c10::nullopt, step, lr, beta1, beta2, eps, wd, bias_correction,
            inst.adamw, 1.0);
  return 0;
}

int destroy_adam(int id) {
  std::lock_guard<std::mutex> lk(g_inst_mu);
  g_instances.erase(id);
  return 0;
}

// ------------------------------------------------------------------ casts
void cast_(torch::Tensor dst, torch::Tensor src, double scale) {
  check_cpu_contig(dst, "dst");
  check_cpu_contig(src, "src");
  TORCH_CHECK(dst.numel() == src.numel(), "size mismatch");
  const void* s = src.data_ptr();
  void* d = dst.data_ptr();
  int sdt = host_dt(src), ddt = host_dt(dst);
  float sc = static_cast<float>(scale);
  pybind11::gil_scoped_release nogil;
  chunked(src.numel(), [&](int64_t b, int64_t e) { cast_range(s, sdt, d, ddt, sc, b, e); });
}

// dst = scale * sum(srcs); every src has dst's numel.  Used by cpu_reduce:
// each rank sums its 1/N slice of all ranks' grad slots.
void sum_slots_(torch::Tensor dst, std::vector<torch::Tensor> srcs, double scale) {
  check_cpu_contig(dst, "dst");
  TORCH_CHECK(!srcs.empty(), "need at least one source");
  std::vector<const void*> ptrs;
  int sdt = host_dt(srcs[0]);
  for (auto& s : srcs) {
    check_cpu_contig(s, "src");
    TORCH_CHECK(s.numel() == dst.numel(), "slot size mismatch");
    TORCH_CHECK(host_dt(s) == sdt, "slot dtypes differ");
    ptrs.push_back(s.data_ptr());
  }
  void* d = dst.data_ptr();
  int ddt = host_dt(dst);
  float sc = static_cast<float>(scale);
  int n = static_cast<int>(ptrs.size());
  pybind11::gil_scoped_release nogil;
  chunked(dst.numel(),
          [&](int64_t b, int64_t e) { sum_slots_range(ptrs.data(), n, sdt, d, ddt, sc, b, e); });
}

double sumsq(torch::Tensor src) {
  check_cpu_contig(src, "src");
  const void* s = src.data_ptr();
  int dt = host_dt(src);
  int64_t n = src.numel();
  int64_t tasks = (n + kChunk - 1) / kChunk;
  std::vector<double> part(tasks > 0 ? tasks : 1, 0.0);
  pybind11::gil_scoped_release nogil;
  ThreadPool::instance().parallel_for(tasks, [&](int64_t t) {
    int64_t b = t * kChunk;
    int64_t e = b + kChunk < n ? b + kChunk : n;
    part[t] = sumsq_range(s, dt, b, e);
  });
  double total = 0.0;
  for (double x : part) total += x;
  return total;
}

// ---------------------------------------------------- shared memory regions
// A region is a file under /dev/shm mapped MAP_SHARED by every local rank.
// It is created sparse with ftruncate (pages materialise as zeros on first
// touch, no explicit zero-fill pass).  The returned tensor keeps the mapping
// alive; the file is unlinked by its creator via shm_unlink().
struct Mapping {
  void* ptr = nullptr;
  size_t bytes = 0;
  ~Mapping() {
    if (ptr && ptr != MAP_FAILED) munmap(ptr, bytes);
  }
};

torch::Tensor shm_map(const std::string& path, int64_t bytes, bool create) {
  TORCH_CHECK(bytes > 0, "shm region must be non-empty");
  int flags = O_RDWR | (create ? (O_CREAT | O_EXCL) : 0);
  int fd = ::open(path.c_str(), flags, 0600);
  TORCH_CHECK(fd >= 0, "open(", path, ") failed: ", std::strerror(errno));
  if (create) {
    if (ftruncate(fd, bytes) != 0) {
      int err = errno;
      ::close(fd);
      TORCH_CHECK(false, "ftruncate(", path, ") failed: ", std::strerror(err));
    }
  } else {
    struct stat st;
    if (fstat(fd, &st) != 0) {
      int err = errno;
      ::close(fd);
      TORCH_CHECK(false, "fstat(", path, ") failed: ", std::strerror(err));
    }
    if (st.st_size < bytes) {
      ::close(fd);
      TORCH_CHECK(false, "shm file ", path, " has ", st.st_size, " bytes, need ", bytes,
                  " (was it created for another model or configuration?)");
    }
  }
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  int err = errno;
  ::close(fd);
  TORCH_CHECK(p != MAP_FAILED, "mmap(", path, ") failed: ", std::strerror(err));
  auto m = std::make_shared<Mapping>();
  m->ptr = p;
  m->bytes = static_cast<size_t>(bytes);
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCPU);
  return torch::from_blob(p, {bytes}, [m](void*) mutable { m.reset(); }, opts);
}

void shm_remove(const std::string& path) { ::unlink(path.c_str()); }

// Anonymous private mapping (single process): the same zero-on-demand
// behaviour, optionally with transparent huge pages.
torch::Tensor anon_map(int64_t bytes, bool hugepages) {
  TORCH_CHECK(bytes > 0, "region must be non-empty");
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  TORCH_CHECK(p != MAP_FAILED, "mmap failed: ", std::strerror(errno));
  if (hugepages) madvise(p, bytes, MADV_HUGEPAGE);
  auto m = std::make_shared<Mapping>();
  m->ptr = p;
  m->bytes = static_cast<size_t>(bytes);
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCPU);
  return torch::from_blob(p, {bytes}, [m](void*) mutable { m.reset(); }, opts);
}

// Touch every page with the calling pool (first-touch placement and avoiding
// page faults inside the timed loop).
void prefault(torch::Tensor region) {
  uint8_t* p = static_cast<uint8_t*>(region.data_ptr());
  int64_t n = region.numel() * region.element_size();
  const int64_t page = 4096;
  pybind11::gil_scoped_release nogil;
  int64_t pages = (n + page - 1) / page;
  int64_t per = 4096;  // pages per task
  ThreadPool::instance().parallel_for((pages + per - 1) / per, [&](int64_t t) {
    int64_t b = t * per * page, e = std::min<int64_t>(n, (t + 1) * per * page);
    for (int64_t i = b; i < e; i += page) {
      volatile uint8_t* q = p + i;
      *q = *q;
    }
  });
}

// Monotonic 64-bit counters living in a shared region (8-byte aligned).
static std::atomic<uint64_t>* counter_at(torch::Tensor& region, int64_t idx) {
  TORCH_CHECK(region.device().is_cpu(), "counter region must be host memory");
  uint8_t* base = static_cast<uint8_t*>(region.data_ptr());
  TORCH_CHECK((idx + 1) * 8 <= region.numel() * region.element_size(), "counter index ", idx,
              " out of range");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 8 == 0, "counter region misaligned");
  return reinterpret_cast<std::atomic<uint64_t>*>(base + idx * 8);
}

uint64_t counter_add(torch::Tensor region, int64_t idx, int64_t delta) {
  return counter_at(region, idx)->fetch_add(static_cast<uint64_t>(delta),
                                            std::memory_order_acq_rel) +
         static_cast<uint64_t>(delta);
}

uint64_t counter_load(torch::Tensor region, int64_t idx) {
  return counter_at(region, idx)->load(std::memory_order_acquire);
}

void counter_store(torch::Tensor region, int64_t idx, int64_t value) {
  counter_at(region, idx)->store(static_cast<uint64_t>(value), std::memory_order_release);
}

// Wait until counter >= target.  Returns false on timeout (never blocks
// longer than timeout_s).  Spins briefly, then sleeps in 20 us steps.
bool counter_wait_geq(torch::Tensor region, int64_t idx, int64_t target, double timeout_s) {
  auto* c = counter_at(region, idx);
  const uint64_t tgt = static_cast<uint64_t>(target);
  if (c->load(std::memory_order_acquire) >= tgt) return true;
  pybind11::gil_scoped_release nogil;
  for (int i = 0; i < 2000; ++i) {
    if (c->load(std::memory_order_acquire) >= tgt) return true;
    __builtin_ia32_pause();
  }
  struct timespec t0;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  struct timespec nap = {0, 20000};
  for (;;) {
    if (c->load(std::memory_order_acquire) >= tgt) return true;
    struct timespec now;
    clock_gettime(CLOCK_MONOTONIC, &now);
    double el = (now.tv_sec - t0.tv_sec) + 1e-9 * (now.tv_nsec - t0.tv_nsec);
    if (el > timeout_s) return false;
    nanosleep(&nap, nullptr);
  }
}

// ------------------------------------------------------------------- NUMA
// mbind(2) through the raw syscall (no libnuma dependency).  mode: "bind",
// "preferred" or "interleave".  Returns 0 or errno (ENOSYS/EPERM in
// containers is tolerated by the caller).
int numa_bind(torch::Tensor region, std::vector<int> nodes, const std::string& mode) {
  if (nodes.empty()) return 0;
  unsigned long mask[16] = {0};
  for (int n : nodes) {
    TORCH_CHECK(n >= 0 && n < 1024, "bad NUMA node ", n);
    mask[n / 64] |= 1ul << (n % 64);
  }
  int pol = mode == "interleave" ? MPOL_INTERLEAVE : mode == "bind" ? MPOL_BIND : MPOL_PREFERRED;
  uintptr_t p = reinterpret_cast<uintptr_t>(region.data_ptr());
  size_t n = region.numel() * region.element_size();
  uintptr_t aligned = p & ~uintptr_t(4095);
  n += p - aligned;
  long rc = syscall(SYS_mbind, aligned, n, pol, mask, 1024, 0);
  return rc == 0 ? 0 : errno;
}

int current_cpu() { return sched_getcpu(); }

}  // namespace t1h

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace t1h;
  m.doc() = "test1_b200 host-side native kernels (LayerAdam, CPU reduce, shm, NUMA)";
  m.def("simd_level", &simd_level);
  m.def("set_simd_level", &set_simd_level);
  m.def("configure_threads", &configure_threads, pybind11::arg("n"),
        pybind11::arg("cpus") = std::vector<int>{});
  m.def("num_threads", &num_threads);
  m.def("adam_step", &adam_step, pybind11::arg("param"), pybind11::arg("grad"),
        pybind11::arg("exp_avg"), pybind11::arg("exp_avg_sq"), pybind11::arg("shadow"),
        pybind11::arg("step"), pybind11::arg("lr"), pybind11::arg("beta1"),
        pybind11::arg("beta2"), pybind11::arg("eps"), pybind11::arg("weight_decay"),
        pybind11::arg("bias_correction") = true, pybind11::arg("adamw_mode") = true,
        pybind11::arg("grad_scale") = 1.0);
  m.def("adam_step_split", &adam_step_split, pybind11::arg("hi"), pybind11::arg("lo"),
        pybind11::arg("grad"), pybind11::arg("exp_avg"), pybind11::arg("exp_avg_sq"),
        pybind11::arg("step"), pybind11::arg("lr"), pybind11::arg("beta1"), pybind11::arg("beta2"),
        pybind11::arg("eps"), pybind11::arg("weight_decay"), pybind11::arg("bias_correction") = true,
        pybind11::arg("adamw_mode") = true, pybind11::arg("grad_scale") = 1.0);
  m.def("f32_to_split", &f32_to_split);
  m.def("split_to_f32", &split_to_f32);
  m.def("create_adam", &create_adam);
  m.def("adam_update", &adam_update);
  m.def("destroy_adam", &destroy_adam);
  m.def("cast_", &cast_, pybind11::arg("dst"), pybind11::arg("src"),
        pybind11::arg("scale") = 1.0);
  m.def("sum_slots_", &sum_slots_, pybind11::arg("dst"), pybind11::arg("srcs"),
        pybind11::arg("scale") = 1.0);
  m.def("sumsq", &sumsq);
  m.def("shm_map", &shm_map);
  m.def("shm_remove", &shm_remove);
  m.def("anon_map", &anon_map, pybind11::arg("bytes"), pybind11::arg("hugepages") = true);
  m.def("prefault", &prefault);
  m.def("counter_add", &counter_add);
  m.def("counter_load", &counter_load);
  m.def("counter_store", &counter_store);
  m.def("counter_wait_geq", &counter_wait_geq);
  m.def("numa_bind", &numa_bind);
  m.def("current_cpu", &current_cpu);
}
