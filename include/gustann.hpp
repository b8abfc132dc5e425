// gustann.hpp -- header-only C++ facade over the C ABI (gann.h) with the
// reference's host API, so a driver written against gustann::GustANN
// (src/ssd_search.hpp:18-83) compiles and links against libgann.so unchanged
// for the in-memory modes. Errors throw std::runtime_error, as the reference's
// CHECK_CUDA does (src/common_cuda.cuh:10-17).
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "gann.h"

namespace gustann {

// src/common.hpp:22-25
enum DataType { UINT8 = 0, FLOAT = 1 };

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

// src/hybrid_config.hpp:8-19; accepted for source compatibility only
struct HybridExecutorConfig {
  int mini_batch = 0;
  int thread_cnt = 0;
  int ctx_per_thread = 0;
  enum { SPDK, MEMORY, URING, AIO } use_backend = MEMORY;
  std::vector<std::string> ssd_lists;
};

class GustANN {
 public:
  explicit GustANN(DataType data_type = FLOAT, int device = 0) : data_type_(data_type), device_(device) {}
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
    check(gann_open(&c, &h_));
  }

  // The SSD-tiered executor (src/hybrid.cu) is not part of this build.
  void init_hybrid(const GustANNConfig&, const HybridExecutorConfig&) {
    throw std::runtime_error("GANN_EUNSUPPORTED: init_hybrid is not provided by this build");
  }

  // src/ssd_search.cu:114-140
  void search(const float* qdata, const int num_queries, const int topk, const int ef_search, int* nns,
              float* distances, int* found_cnt, GustANNStats* stats = nullptr) {
    if (!h_) throw std::runtime_error("GANN_ESTATE: search before init_pure_mem");
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
  static void check(int rc) {
    if (rc != GANN_OK) throw std::runtime_error(std::string("gann error ") + std::to_string(rc) + ": " + gann_last_error());
  }
  DataType data_type_;
  int device_;
  gann_handle* h_ = nullptr;
};

}  // namespace gustann
