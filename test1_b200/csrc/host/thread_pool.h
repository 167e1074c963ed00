// Persistent worker pool for the host-side hot loops (LayerAdam, CPU reduce,
// casts).  One pool per process; workers can be pinned to an explicit CPU
// list so that each rank's optimizer threads stay on the NUMA node of its
// GPU.  OpenMP is deliberately not used: torchrun sets OMP_NUM_THREADS=1 for
// every rank, and the pool must be sized and pinned per rank at run time.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace t1h {

class ThreadPool {
 public:
  static ThreadPool& instance();

  // (Re)create `n` workers.  `cpus` (may be empty) lists the CPUs the workers
  // are pinned to, round-robin.  The calling thread also executes tasks.
  void configure(int n, const std::vector<int>& cpus);
  int num_threads() const { return static_cast<int>(workers_.size()) + 1; }

  // Run fn(task) for task in [0, n_tasks).  Blocks until all tasks finished.
  // Calls from different threads are serialised.
  void parallel_for(int64_t n_tasks, const std::function<void(int64_t)>& fn);

  ~ThreadPool();

 private:
  ThreadPool() = default;
  void stop_workers();
  void worker_loop(int idx, int cpu, uint64_t start_generation);
  void run_tasks();

  std::vector<std::thread> workers_;
  std::mutex job_mutex_;   // serialises parallel_for callers
  std::mutex mu_;
  std::condition_variable cv_start_;
  std::condition_variable cv_done_;
  uint64_t generation_ = 0;
  bool stopping_ = false;
  int active_ = 0;  // workers still inside the current job

  const std::function<void(int64_t)>* fn_ = nullptr;
  int64_t n_tasks_ = 0;
  std::atomic<int64_t> next_task_{0};
};

}  // namespace t1h
