#include "thread_pool.h"

#include <pthread.h>
#include <sched.h>

namespace t1h {

ThreadPool& ThreadPool::instance() {
  static ThreadPool pool;
  return pool;
}

ThreadPool::~ThreadPool() { stop_workers(); }

void ThreadPool::stop_workers() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stopping_ = true;
    ++generation_;
  }
  cv_start_.notify_all();
  for (auto& t : workers_) {
    if (t.joinable()) t.join();
  }
  workers_.clear();
  std::lock_guard<std::mutex> lk(mu_);
  stopping_ = false;
}

void ThreadPool::configure(int n, const std::vector<int>& cpus) {
  std::lock_guard<std::mutex> job(job_mutex_);
  stop_workers();
  int extra = n > 1 ? n - 1 : 0;
  uint64_t gen;
  {
    std::lock_guard<std::mutex> lk(mu_);
    gen = generation_;
  }
  // Each worker starts from the generation current *now*, so a job posted
  // before the thread gets scheduled is not missed.
  for (int i = 0; i < extra; ++i) {
    int cpu = cpus.empty() ? -1 : cpus[(i + 1) % cpus.size()];
    workers_.emplace_back(&ThreadPool::worker_loop, this, i, cpu, gen);
  }
  if (!cpus.empty()) {
    // The calling thread takes the first CPU of the list only while it runs
    // tasks; it is not re-pinned permanently (it is usually a Python thread).
  }
}

void ThreadPool::run_tasks() {
  const auto& fn = *fn_;
  for (;;) {
    int64_t t = next_task_.fetch_add(1, std::memory_order_relaxed);
    if (t >= n_tasks_) break;
    fn(t);
  }
}

void ThreadPool::worker_loop(int /*idx*/, int cpu, uint64_t start_generation) {
  if (cpu >= 0) {
    cpu_set_t set;
    CPU_ZERO(&set);
    CPU_SET(cpu, &set);
    pthread_setaffinity_np(pthread_self(), sizeof(set), &set);
  }
  uint64_t seen = start_generation;
  for (;;) {
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_start_.wait(lk, [&] { return generation_ != seen; });
      seen = generation_;
      if (stopping_) return;
    }
    run_tasks();
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (--active_ == 0) cv_done_.notify_all();
    }
  }
}

void ThreadPool::parallel_for(int64_t n_tasks, const std::function<void(int64_t)>& fn) {
  if (n_tasks <= 0) return;
  std::lock_guard<std::mutex> job(job_mutex_);
  if (workers_.empty() || n_tasks == 1) {
    for (int64_t t = 0; t < n_tasks; ++t) fn(t);
    return;
  }
  {
    std::lock_guard<std::mutex> lk(mu_);
    fn_ = &fn;
    n_tasks_ = n_tasks;
    next_task_.store(0, std::memory_order_relaxed);
    active_ = static_cast<int>(workers_.size());
    ++generation_;
  }
  cv_start_.notify_all();
  run_tasks();
  std::unique_lock<std::mutex> lk(mu_);
  cv_done_.wait(lk, [&] { return active_ == 0; });
  fn_ = nullptr;
}

}  // namespace t1h
