// gustann.hpp -- header-only C++ facade over the C ABI (gann.h) with the
// reference's host API, so a driver written against gustann::GustANN
// (src/ssd_search.hpp:18-83) compiles and links against libgann.so unchanged
// for the in-memory and hybrid modes. Errors throw std::runtime_error, as the reference's
// CHECK_CUDA does (src/common_cuda.cuh:10-17).
#pragma once

#include <chrono>
#include <future>
#include <stdexcept>
#include <string>
#include <vector>

#include "gann.h"

namespace gustann {

// src/common.hpp:22-25
enum DataType { UINT8 = 0, FLOAT = 1 };

// Distance (an extension: the reference is L2-only, src/common.hpp:28-30).
enum Metric { L2 = GANN_METRIC_L2, INNER_PRODUCT = GANN_METRIC_IP };

// src/ssd_search.hpp:18-23
class GustANNConfig {
 public:
  std::string index_file;
  std::string pq_file_prefix;
  std::string nav_graph_prefix;
};

// src/ssd_search.hpp:25-27 (run_time), plus the counters gann_stats adds
struct GustANNStats {
  double run_time = 0.0;
  double total_time = 0.0;
  long long hops = 0;
  long long adc_evals = 0;
  long long capped_queries = 0;
  long long bytes_touched = 0;
};

// src/hybrid_config.hpp:8-19. mini_batch (> 0: queries per hop batch),
// thread_cnt (page reader threads) and ctx_per_thread (mini-batches in flight,
// whose page reads overlap each other's GPU hops) are used; the IO backend is
// always a threaded pread of the local index file (src/io/mem_io.cpp's role).
struct HybridExecutorConfig {
  int mini_batch = 0;
  int thread_cnt = 0;
  int ctx_per_thread = 0;
  enum { SPDK, MEMORY, URING, AIO } use_backend = MEMORY;
  std::vector<std::string> ssd_lists;
};

class GustANN {
 public:
  explicit GustANN(DataType data_type = FLOAT, int device = 0, Metric metric = L2)
      : data_type_(data_type), device_(device), metric_(metric) {}
  GustANN(const GustANN&) = delete;
  GustANN& operator=(const GustANN&) = delete;
  ~GustANN() { gann_close(h_); }

  // src/ssd_search.cu:108-112
  void init_pure_mem(const GustANNConfig& config, bool use_gpu_mem) {
    gann_close(h_);
    h_ = nullptr;
    gann_config c{};
    c.index_file = config.index_file.c_str();
    c.pq_file_prefix = config.pq_file_prefix.c_str();
    c.nav_graph_prefix = config.nav_graph_prefix.c_str();
    c.dtype = data_type_;
    c.use_gpu_mem = use_gpu_mem ? 1 : 0;
    c.device = device_;
    c.metric = metric_;
    check(gann_open(&c, &h_));
    is_hybrid_ = false;
  }

  // src/ssd_search.cu:81-106: node records stay in the index file; search()
  // then drives the host-driven hop search (gann_hop_*), reading the page of
  // every query's next node between hops.
  void init_hybrid(const GustANNConfig& config, const HybridExecutorConfig& hc) {
    gann_close(h_);
    h_ = nullptr;
    index_file_ = config.index_file;
    gann_config c{};
    c.index_file = config.index_file.c_str();
    c.pq_file_prefix = config.pq_file_prefix.c_str();
    c.nav_graph_prefix = config.nav_graph_prefix.c_str();
    c.dtype = data_type_;
    c.use_gpu_mem = 2;
    c.device = device_;
    c.metric = metric_;
    check(gann_open(&c, &h_));
    hybrid_ = hc;
    is_hybrid_ = true;
  }

  // src/ssd_search.cu:114-140
  void search(const float* qdata, const int num_queries, const int topk, const int ef_search, int* nns,
              float* distances, int* found_cnt, GustANNStats* stats = nullptr) {
    if (!h_) throw std::runtime_error("GANN_ESTATE: search before init_pure_mem");
    if (is_hybrid_) {
      search_hybrid(qdata, num_queries, topk, ef_search, nns, distances, found_cnt, stats);
      return;
    }
    gann_stats st{};
    check(gann_search(h_, qdata, num_queries, topk, ef_search, nns, distances, found_cnt, &st));
    if (stats) {
      stats->run_time = st.run_time;
      stats->total_time = st.total_time;
      stats->hops = st.hops;
      stats->adc_evals = st.adc_evals;
      stats->capped_queries = st.capped_queries;
      stats->bytes_touched = st.bytes_touched;
    }
  }

  gann_handle* handle() const { return h_; }

 private:
  // Mini-batches of `mini_batch` queries, `ctx_per_thread` of them in flight
  // (src/hybrid.cu:56-58,82-83: contexts per reader thread). With one, each
  // round reads the pages of the batch's next nodes, then runs its hop. With
  // K >= 2 the batches take turns: while batch i's hop runs on the GPU, a
  // second host thread reads the pages batch i+1 (mod K) asked for, so page
  // reads and GPU steps overlap. Every batch is independent, so results do
  // not depend on K.
  struct HopSlot {
    gann_hop_batch* b = nullptr;
    int lo = 0, n = 0;
    int64_t active = 0;
    std::vector<int32_t> ids;
    std::vector<unsigned char> pages;
  };

  void search_hybrid(const float* qdata, int nq, int topk, int ef, int* nns, float* distances, int* found_cnt,
                     GustANNStats* stats) {
    const auto t0 = std::chrono::steady_clock::now();
    gann_info info{};
    check(gann_index_info(h_, &info));
    const int batch = hybrid_.mini_batch > 0 ? hybrid_.mini_batch : (nq > 0 ? nq : 1);
    const int k = hybrid_.ctx_per_thread > 1 ? hybrid_.ctx_per_thread : 1;
    std::vector<HopSlot> slot(static_cast<size_t>(k));
    int next = 0;
    long long hops = 0;
    // the next mini-batch into slot s, with its entry nodes requested
    auto open = [&](HopSlot& s) -> int {
      s.b = nullptr;
      s.active = 0;
      if (next >= nq) return GANN_OK;
      s.lo = next;
      s.n = nq - next < batch ? nq - next : batch;
      next += s.n;
      int rc = gann_hop_begin(h_, qdata + static_cast<size_t>(s.lo) * info.dim, s.n, topk, ef, &s.b);
      if (rc != GANN_OK) return rc;
      s.ids.assign(static_cast<size_t>(s.n), -1);
      s.pages.assign(static_cast<size_t>(s.n) * 4096, 0);
      return gann_hop_requests(s.b, s.ids.data(), &s.active);
    };
    auto read = [&](HopSlot& s) -> int {
      return s.b && s.active ? gann_read_pages(index_file_.c_str(), s.ids.data(), s.n, info.nodes_per_page,
                                               s.pages.data(), hybrid_.thread_cnt)
                             : GANN_OK;
    };
    // one hop of slot s (its pages already read); a finished batch writes its
    // results and the slot takes the next one
    auto step = [&](HopSlot& s) -> int {
      if (!s.b) return GANN_OK;
      int rc = GANN_OK;
      if (s.active) {
        if ((rc = gann_hop_step(s.b, s.pages.data())) != GANN_OK) return rc;
        ++hops;
        if ((rc = gann_hop_requests(s.b, s.ids.data(), &s.active)) != GANN_OK) return rc;
      }
      if (s.active) return GANN_OK;
      rc = gann_hop_finish(s.b, nns + static_cast<size_t>(s.lo) * topk, distances + static_cast<size_t>(s.lo) * topk,
                           found_cnt + s.lo);
      gann_hop_free(s.b);
      s.b = nullptr;
      return rc != GANN_OK ? rc : open(s);
    };
    auto any_open = [&]() {
      for (const HopSlot& s : slot)
        if (s.b) return true;
      return false;
    };
    auto fail = [&](int rc) {
      for (HopSlot& s : slot)
        if (s.b) gann_hop_free(s.b);
      check(rc);
    };
    int rc = GANN_OK;
    for (HopSlot& s : slot)
      if ((rc = open(s)) != GANN_OK) fail(rc);
    if (k == 1) {
      while (slot[0].b) {
        if ((rc = read(slot[0])) != GANN_OK || (rc = step(slot[0])) != GANN_OK) fail(rc);
      }
    } else {
      if ((rc = read(slot[0])) != GANN_OK) fail(rc);
      for (int cur = 0; any_open(); cur = (cur + 1) % k) {
        HopSlot& nx = slot[static_cast<size_t>((cur + 1) % k)];
        std::future<int> pending = std::async(std::launch::async, [&]() { return read(nx); });
        const int rs = step(slot[static_cast<size_t>(cur)]);
        const int rr = pending.get();
        if (rs != GANN_OK || rr != GANN_OK) fail(rs != GANN_OK ? rs : rr);
      }
    }
    if (stats) {
      *stats = GustANNStats();
      // wall time of the whole hop loop: entry search, page reads and hops
      stats->run_time = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      stats->total_time = stats->run_time;
      stats->hops = hops;   // hop rounds (one page read per active query each)
    }
  }

  static void check(int rc) {
    if (rc != GANN_OK) throw std::runtime_error(std::string("gann error ") + std::to_string(rc) + ": " + gann_last_error());
  }
  DataType data_type_;
  int device_;
  Metric metric_ = L2;
  gann_handle* h_ = nullptr;
  bool is_hybrid_ = false;
  HybridExecutorConfig hybrid_;
  std::string index_file_;
};

}  // namespace gustann
