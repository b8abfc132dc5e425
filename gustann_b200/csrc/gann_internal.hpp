// Internal structures shared by the loader, the C ABI and the kernels.
#pragma once

#include <cstdint>
#include <cstddef>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "gann.h"

namespace gann {

constexpr int kWarp = 32;
constexpr int kPivots = 256;            // PQSearchData::num_pivots (src/pq_search.hpp:12)
constexpr uint32_t kPadId = 0xffffffffu;
constexpr uint32_t kVisited = 0x80000000u;
constexpr int kNavSlots = 32;           // nav pool: 4 best + 28 neighbour slots
constexpr int kNavBest = 4;             // src/impl/nav.cuh:11
constexpr int kNavNbr = 28;             // src/impl/nav.cuh:12
constexpr int kPageSize = 4096;

// Host-side copy of everything parsed from the three index inputs.
struct HostIndex {
  int dtype = GANN_FLOAT;
  int elem = 4;
  // disk index header (src/layout.cpp:25-54)
  int64_t num_points = 0, dim = 0, medoid = 0;
  int64_t max_node_len = 0, nodes_per_page = 0, max_m0 = 0, data_size = 0, num_pages = 0;
  // PQ (src/pq_search.cu:56-121)
  int num_chunks = 0;
  std::vector<float> pivots_t;          // [dim x 256], transposed like the reference
  std::vector<float> centroid;          // [dim]
  std::vector<int32_t> chunk_offsets;   // [M+1]
  // nav graph (src/nav_graph.cu:41-100)
  bool has_nav = false;
  int64_t nav_points = 0;
  int32_t nav_max_m = 0, nav_start = 0;
  std::vector<uint8_t> nav_vecs;        // [S x nav_stride] bytes
  std::vector<int32_t> nav_adj;         // [S x nav_max_m] + 32 tail, -1 padded
  std::vector<int32_t> nav_map;         // [S]
};

// Device layout: records split into aligned vector rows and adjacency rows.
constexpr int kMaxParts = 8;

struct DeviceIndex {
  const uint8_t* vecs = nullptr;     // [N x vec_stride]
  const uint32_t* adj = nullptr;     // [N x adj_stride] u32, kPadId after deg
  const uint8_t* codes = nullptr;    // [N x code_stride]
  const float* pivots_t = nullptr;   // [D x 256]
  const float* centroid = nullptr;   // [D]
  const int32_t* chunk_off = nullptr;// [M+1]
  const uint8_t* nav_vecs = nullptr; // [S x nav_stride]
  const int32_t* nav_adj = nullptr;  // [S x nav_row] + 32 tail, -1 padded
  const int32_t* nav_map = nullptr;  // [S]
  int64_t n = 0;
  int32_t dim = 0, degree = 0, chunks = 0;
  int64_t vec_stride = 0;            // bytes, multiple of 32 elements
  int32_t adj_stride = 0;            // u32 words
  int32_t code_stride = 0;           // bytes, multiple of 16
  int64_t nav_stride = 0;            // bytes
  int32_t nav_start = 0, has_nav = 0, nav_row = 0;
  int64_t nav_points = 0;
  int64_t medoid = 0;
  // pivot table [M x 256] float4, chunk dims zero-padded to 4; piv_width = 3
  // when every chunk has 3 dims, 4 when all have <= 4, 0 when a chunk is wider
  const float4* piv4 = nullptr;
  int32_t piv_width = 0;
  // neighbour-code layout: row u = the code rows of adj[u][0..adj_stride),
  // each code_stride bytes (nullptr when the index keeps codes separate only)
  const uint8_t* ncodes = nullptr;
  int32_t adc_mode = 0;     // 0 auto, 1 table, 2 pivot
  int32_t metric = 0;       // GANN_METRIC_L2 / GANN_METRIC_IP
  int32_t piv_warps = 0;    // 0 = as many as fit (<= 24)
  // records split by id (nparts > 1): part p holds ids [p << part_shift,
  // (p + 1) << part_shift) in its own arrays (possibly another GPU's memory,
  // reached through peer pointers); vecs/adj/ncodes above are then unused
  int32_t nparts = 0;
  int32_t part_shift = 0;
  int32_t local_part = -1;  // the range in this GPU's memory (-1: every range)
  const uint8_t* part_vecs[kMaxParts] = {};
  const uint32_t* part_adj[kMaxParts] = {};
  const uint8_t* part_ncodes[kMaxParts] = {};
};

struct SearchArgs {
  const float* q = nullptr;
  int64_t nq = 0;
  int32_t topk = 0, ef = 0;
  int32_t max_hops = 0, nav_max_hops = 0;
  int32_t* nns = nullptr;
  float* dist = nullptr;
  int32_t* found = nullptr;
  uint32_t* hops = nullptr;        // nullable
  uint32_t* adc = nullptr;         // nullable
  int32_t* qcounter = nullptr;     // work counter (zeroed before launch)
  int32_t* err = nullptr;          // [2]: capped queries, capped nav searches
  // per-warp visited-id tables (nullable): vis_slots tables of 2^kVisBits ids,
  // table i used by the warp with global warp index i
  uint32_t* vis = nullptr;
  int64_t vis_slots = 0;
};

// Visited-id table of one warp: 2^kVisBits slots (8 KB). A buffer of
// sm_count * kVisWarpsPerSM tables covers every warp either kernel keeps
// resident (at most 32 one-warp CTAs per SM in table mode).
constexpr int kVisBits = 11;
constexpr int kVisWarpsPerSM = 32;

// Host-driven search, one hop per call: the reference's SSD-hybrid mode
// (src/hyd_task_runner.cu, src/impl/hyd_search_v2.cuh), in which the caller
// fetches the 4 KB page of every query's next node between hops. Per-query
// state lives in device memory between calls.
struct HopState {
  int64_t nq = 0;
  int32_t topk = 0, ef = 0, max_hops = 0, nav_max_hops = 0;
  float* qpp = nullptr;       // [nq x dim] q'' = (q - c) + c
  float* lut = nullptr;       // [nq x M x 256] ADC tables
  uint64_t* pool = nullptr;   // [nq x ef] keys (see gann_search.cu)
  int32_t* psize = nullptr;   // [nq]
  int32_t* request = nullptr; // [nq] node expanded next, -1 when done
  int32_t* nns = nullptr;     // [nq x topk]
  float* dist = nullptr;      // [nq x topk]
  int32_t* found = nullptr;   // [nq]
  uint32_t* hops = nullptr;   // [nq]
  int32_t* err = nullptr;     // [3]: capped queries, capped nav searches, bad records
};

// Kernel launchers (gann_search.cu)
cudaError_t launch_hop_begin(const DeviceIndex& ix, const float* d_q, const HopState& s, int dtype,
                             cudaStream_t st);
cudaError_t launch_hop_step(const DeviceIndex& ix, const HopState& s, const uint8_t* d_pages, int32_t node_len,
                            int32_t nodes_per_page, int dtype, cudaStream_t st);
cudaError_t launch_search(const DeviceIndex& ix, const SearchArgs& a, int dtype,
                          int sm_count, cudaStream_t st);
cudaError_t launch_probe_lut(const DeviceIndex& ix, const float* d_q, int64_t nq,
                             float* d_lut, cudaStream_t st);
cudaError_t launch_probe_entry(const DeviceIndex& ix, const float* d_q, int64_t nq,
                               int dtype, int32_t* d_sample, int32_t* d_entry,
                               int32_t* d_err, cudaStream_t st);
size_t search_smem_bytes(const DeviceIndex& ix, int topk, int ef);
// Pivot table of the pivot-mode kernel from the [256 x dim] PQ pivots; returns
// the width code (see DeviceIndex::piv_width) and fills `out` when it is > 0.
int make_pivot_table(const std::vector<float>& pivots_t, const std::vector<int32_t>& chunk_off, int dim,
                     std::vector<float>& out);
int search_max_ef();
// RobustPrune for the GPU index builder (gann_build.cu).
int prune_max_candidates();
cudaError_t launch_sort_unique_rows(const int32_t* ids, const float* dists, int64_t rows, int k, int32_t* out_ids,
                                    float* out_d, int sm_count, cudaStream_t st);
cudaError_t launch_robust_prune(const void* vecs, int64_t n, int64_t stride, int dim, int dtype,
                                const int32_t* points, int64_t b, const int32_t* cand, const float* cdist, int k,
                                int r, float alpha, int32_t* out, float* outd, int sm_count, cudaStream_t st);
// Exact brute-force k-NN (gann_exact.cu).
int exact_knn_max_k();
cudaError_t launch_exact_knn(const void* base, int64_t n, int64_t bstride, int dim, int dtype, const void* queries,
                             int64_t qstride, int64_t nq, int k, int metric, int32_t* ids, float* dists,
                             int sm_count, cudaStream_t st);
cudaError_t launch_gather_neighbour_codes(const uint32_t* adj, int adj_stride, int degree, const uint8_t* codes,
                                          int code_stride, int64_t n, uint8_t* out, cudaStream_t st);

// Loader (gann_loader.cpp). Return GANN_* and fill `msg` on error.
int load_disk_header(const std::string& path, int elem, HostIndex& hi, std::string& msg);
int load_pq(const std::string& prefix, HostIndex& hi, std::vector<uint8_t>& codes,
            int64_t& code_rows, std::string& msg);
int load_nav(const std::string& dir, HostIndex& hi, std::string& msg);
// Read records [first, first+count) of the disk index and split them into
// vector rows and padded adjacency rows; validates degrees and ids.
int relayout_records(const std::string& path, const HostIndex& hi, int64_t first, int64_t count,
                     uint8_t* vec_out, int64_t vec_stride, uint32_t* adj_out, int32_t adj_stride,
                     std::string& msg);

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

}  // namespace gann
