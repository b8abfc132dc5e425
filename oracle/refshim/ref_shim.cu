// TEST INFRASTRUCTURE: a C-ABI shim over the reference's own search library,
// compiled (from the reference sources where they lie) into
// oracle/_ref/libgustann_ref.so by oracle/Makefile. It lets the parity tests
// run the reference's unmodified kernels on the B200 next to this build.
//
// Entry points drive the reference's public API and objects:
//   ref_open/ref_search   gustann::GustANN::init_pure_mem + search
//                         (src/ssd_search.hpp:29-83)
//   ref_lut               PQSearchData::init_query via PQSearch
//                         (src/impl/pq.cuh:8-59, src/pq_search.cu:56-185)
//   ref_nav               get_entry_kernel + NavGraph::translate
//                         (src/impl/nav.cuh:13-135, src/nav_graph.cu:41-109)
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "ssd_search.hpp"
#include "pq_search.hpp"
#include "nav_graph.hpp"
#include "impl/pq.cuh"
#include "impl/nav.cuh"

namespace {

struct RefHandle {
  gustann::GustANN* g = nullptr;
  std::string index, pq, nav;
  int dtype = 1;
};

__global__ void ref_lut_kernel(gustann::PQSearchData* pq, float* q, int dim) {
  pq->init_query(q + static_cast<size_t>(blockIdx.x) * dim);
}

int check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "ref_shim: %s: %s\n", what, cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

}  // namespace

extern "C" {

void* ref_open(const char* index_file, const char* pq_prefix, const char* nav_dir, int dtype, int use_gpu_mem) {
  RefHandle* h = new RefHandle();
  h->index = index_file;
  h->pq = pq_prefix;
  h->nav = nav_dir ? nav_dir : "";
  h->dtype = dtype;
  gustann::GustANNConfig cfg;
  cfg.index_file = h->index;
  cfg.pq_file_prefix = h->pq;
  cfg.nav_graph_prefix = h->nav;
  h->g = new gustann::GustANN(dtype == 0 ? gustann::UINT8 : gustann::FLOAT);
  h->g->init_pure_mem(cfg, use_gpu_mem != 0);
  return h;
}

int ref_search(void* hp, const float* q, int nq, int topk, int ef, int* nns, float* dist, int* found,
               double* run_time) {
  RefHandle* h = static_cast<RefHandle*>(hp);
  gustann::GustANNStats st{0.0};
  h->g->search(q, nq, topk, ef, nns, dist, found, &st);
  if (run_time) *run_time = st.run_time;
  return check(cudaGetLastError(), "search");
}

// Per-query ADC tables [nq x M x 256] computed by the reference's device code.
int ref_lut(void* hp, const float* q, int nq, int dim, float* out) {
  RefHandle* h = static_cast<RefHandle*>(hp);
  gustann::PQSearch pq;
  pq.read_data(h->pq + "_pivots.bin", h->pq + "_compressed.bin");
  const int m = pq.get_data().num_chunks;
  pq.init_device(dim, pq.get_data().num_pts, nq, 0);
  float* dq = nullptr;
  if (check(cudaMalloc(&dq, sizeof(float) * nq * dim), "malloc")) return -1;
  cudaMemcpy(dq, q, sizeof(float) * nq * dim, cudaMemcpyHostToDevice);
  ref_lut_kernel<<<nq, 64>>>(pq.get_device_ptr(), dq, dim);
  if (check(cudaDeviceSynchronize(), "lut kernel")) return -1;
  cudaMemcpy(out, pq.device_data.pq_dists, sizeof(float) * nq * m * gustann::PQSearchData::num_pivots,
             cudaMemcpyDeviceToHost);
  cudaFree(dq);
  return check(cudaGetLastError(), "lut copy");
}

// Nav entry per query: sample index and translated global id.
int ref_nav(void* hp, const float* q, int nq, int dim, int* sample, int* entry) {
  RefHandle* h = static_cast<RefHandle*>(hp);
  const int dsize = h->dtype == 0 ? 1 : 4;
  gustann::NavGraph nav;
  nav.init(h->nav + "/nav_index", h->nav + "/nav_index.data", h->nav + "/map.txt", dsize);
  float* dq = nullptr;
  int* dres = nullptr;
  if (check(cudaMalloc(&dq, sizeof(float) * nq * dim), "malloc")) return -1;
  if (check(cudaMalloc(&dres, sizeof(int) * nq), "malloc")) return -1;
  cudaMemcpy(dq, q, sizeof(float) * nq * dim, cudaMemcpyHostToDevice);
  gustann::get_entry_kernel(h->dtype == 0 ? gustann::UINT8 : gustann::FLOAT)<<<(nq + 1) / 2, 64>>>(
      dq, nav.data_dev, nav.graph_dev, nq, nav.num_node, dim, nav.max_m, 5, nav.start, dres, nullptr, nullptr);
  if (check(cudaDeviceSynchronize(), "nav kernel")) return -1;
  cudaMemcpy(sample, dres, sizeof(int) * nq, cudaMemcpyDeviceToHost);
  std::memcpy(entry, sample, sizeof(int) * nq);
  nav.translate(entry, nq);
  cudaFree(dq);
  cudaFree(dres);
  return 0;
}

void ref_close(void* hp) {
  RefHandle* h = static_cast<RefHandle*>(hp);
  delete h->g;
  delete h;
}

}  // extern "C"
