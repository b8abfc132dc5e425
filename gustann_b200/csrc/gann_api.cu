// C ABI of libgann.so: index load onto one B200, search orchestration, stage
// probes. See include/gann.h for the contract of every entry point.
#include <algorithm>
#include <unistd.h>
#include <fcntl.h>
#include <thread>
#include <atomic>
#include <chrono>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "gann_internal.hpp"

using gann::DeviceIndex;
using gann::HostIndex;

namespace {

thread_local std::string g_last_error;

int set_error(int code, const std::string& m) {
  g_last_error = m;
  return code;
}

#define GANN_CUDA(call)                                                                          \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess)                                                                       \
      return set_error(e_ == cudaErrorMemoryAllocation ? GANN_ENOMEM : GANN_ECUDA,               \
                       std::string("CUDA error: ") + cudaGetErrorString(e_) + " (" #call ")"); \
  } while (0)

template <typename T>
int dev_upload(T*& dst, const T* src, size_t count, int64_t& bytes) {
  if (count == 0) return GANN_OK;
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&dst), sizeof(T) * count));
  bytes += static_cast<int64_t>(sizeof(T) * count);
  GANN_CUDA(cudaMemcpy(dst, src, sizeof(T) * count, cudaMemcpyHostToDevice));
  return GANN_OK;
}

}  // namespace

struct gann_handle {
  int device = 0;
  int dtype = GANN_FLOAT;
  bool host_records = false;
  bool storage_records = false;      // records left on storage (host-driven hops only)
  bool cuda_ready = false;           // a CUDA context exists for `device`
  bool owns_records = true;          // false: vectors/adjacency/codes belong to the caller
  HostIndex hi;
  DeviceIndex ix;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  // owned allocations
  uint8_t* vecs = nullptr;
  uint32_t* adj = nullptr;
  uint8_t* codes = nullptr;
  float* pivots_t = nullptr;
  float* centroid = nullptr;
  int32_t* chunk_off = nullptr;
  float* piv4 = nullptr;
  uint8_t* ncodes = nullptr;         // neighbour-code copy (layout 0/2)
  uint8_t* nav_vecs = nullptr;
  int32_t* nav_adj = nullptr;
  int32_t* nav_map = nullptr;
  int32_t* counter = nullptr;        // [0]: work counter, [1..2]: error counts
  uint32_t* vis = nullptr;           // per-warp visited-id tables
  int64_t vis_slots = 0;
  const uint8_t* ncodes_on = nullptr;  // ix.ncodes value when the copy is in use
  // split records (part_count > 1): this handle's ranges, or ranges mapped
  // from other processes (pattached)
  int32_t part_count = 0, part_index = 0;
  int32_t part_ncodes = 0;           // every range carries neighbour codes
  uint8_t* pvecs[gann::kMaxParts] = {};
  uint32_t* padj[gann::kMaxParts] = {};
  uint8_t* pncodes[gann::kMaxParts] = {};
  bool ppresent[gann::kMaxParts] = {};
  bool pattached[gann::kMaxParts] = {};
  int64_t device_bytes = 0;
  // reusable buffers of gann_search
  int64_t cap_q = 0, cap_out = 0;
  float* d_q = nullptr;
  int32_t* d_nns = nullptr;
  float* d_dist = nullptr;
  int32_t* d_found = nullptr;
  uint32_t* d_hops = nullptr;
  uint32_t* d_adc = nullptr;

  void release() {
    if (!cuda_ready) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (!owns_records) {
      vecs = nullptr;
      adj = nullptr;
      codes = nullptr;
    } else if (host_records) {
      if (vecs) cudaFreeHost(vecs);
      if (adj) cudaFreeHost(adj);
    } else {
      if (vecs) cudaFree(vecs);
      if (adj) cudaFree(adj);
    }
    for (void* p : {static_cast<void*>(codes), static_cast<void*>(pivots_t), static_cast<void*>(centroid),
                    static_cast<void*>(chunk_off), static_cast<void*>(piv4), static_cast<void*>(ncodes),
                    static_cast<void*>(nav_vecs), static_cast<void*>(nav_adj),
                    static_cast<void*>(nav_map), static_cast<void*>(counter), static_cast<void*>(vis),
                    static_cast<void*>(d_q),
                    static_cast<void*>(d_nns), static_cast<void*>(d_dist), static_cast<void*>(d_found),
                    static_cast<void*>(d_hops), static_cast<void*>(d_adc)})
      if (p) cudaFree(p);
    for (int p = 0; p < gann::kMaxParts; ++p) {
      for (void* q : {static_cast<void*>(pvecs[p]), static_cast<void*>(padj[p]), static_cast<void*>(pncodes[p])}) {
        if (!q) continue;
        if (pattached[p]) cudaIpcCloseMemHandle(q);
        else cudaFree(q);
      }
      pvecs[p] = nullptr;
      padj[p] = nullptr;
      pncodes[p] = nullptr;
    }
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (stream) cudaStreamDestroy(stream);
    vecs = nullptr;
    adj = nullptr;
    cudaSetDevice(prev);
  }
};

namespace {

// Visited-id tables for every warp the search kernels keep resident. The
// search skips neighbours whose id is in its warp's table; the table is
// cleared per query (by the kernel), so no state crosses queries or calls.
cudaError_t alloc_vis(gann_handle* h) {
  h->vis_slots = static_cast<int64_t>(h->sm_count) * gann::kVisWarpsPerSM;
  const size_t bytes = sizeof(uint32_t) * (static_cast<size_t>(h->vis_slots) << gann::kVisBits);
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&h->vis), bytes);
  if (e != cudaSuccess) {
    h->vis = nullptr;
    h->vis_slots = 0;
    return e;
  }
  h->device_bytes += static_cast<int64_t>(bytes);
  return cudaSuccess;
}

int load_records(gann_handle* h, const std::string& path) {
  HostIndex& hi = h->hi;
  const int64_t n = hi.num_points;
  const int64_t vs = gann::round_up(hi.dim, 32) * hi.elem;
  const int32_t as = static_cast<int32_t>(gann::round_up(hi.max_m0, 4));
  const size_t vbytes = static_cast<size_t>(n) * vs, abytes = static_cast<size_t>(n) * as * 4;
  std::string msg;
  if (h->host_records) {
    // records stay in pinned host memory and are read by the kernel through
    // the unified address space (the reference's search_graph_kernel_dram mode)
    GANN_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->vecs), vbytes, cudaHostAllocMapped | cudaHostAllocPortable));
    GANN_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->adj), abytes, cudaHostAllocMapped | cudaHostAllocPortable));
    const int64_t blk = 1 << 20;
    for (int64_t r = 0; r < n; r += blk) {
      const int64_t c = std::min(blk, n - r);
      int rc = gann::relayout_records(path, hi, r, c, h->vecs + r * vs, vs, h->adj + r * as, as, msg);
      if (rc) return set_error(rc, msg);
    }
  } else {
    GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->vecs), vbytes));
    GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->adj), abytes));
    h->device_bytes += static_cast<int64_t>(vbytes + abytes);
    const int64_t blk = 1 << 20;
    std::vector<uint8_t> sv(static_cast<size_t>(std::min(blk, n)) * vs);
    std::vector<uint32_t> sa(static_cast<size_t>(std::min(blk, n)) * as);
    for (int64_t r = 0; r < n; r += blk) {
      const int64_t c = std::min(blk, n - r);
      int rc = gann::relayout_records(path, hi, r, c, sv.data(), vs, sa.data(), as, msg);
      if (rc) return set_error(rc, msg);
      GANN_CUDA(cudaMemcpy(h->vecs + r * vs, sv.data(), static_cast<size_t>(c) * vs, cudaMemcpyHostToDevice));
      GANN_CUDA(cudaMemcpy(h->adj + r * as, sa.data(), static_cast<size_t>(c) * as * 4, cudaMemcpyHostToDevice));
    }
  }
  h->ix.vecs = h->vecs;
  h->ix.adj = h->adj;
  h->ix.vec_stride = vs;
  h->ix.adj_stride = as;
  return GANN_OK;
}

// Split records: id range p = [p << shift, (p + 1) << shift) of the index,
// with its own vector, adjacency and (when it fits) neighbour-code arrays.
int load_part(gann_handle* h, const gann_config* cfg, int p, bool with_ncodes) {
  HostIndex& hi = h->hi;
  DeviceIndex& ix = h->ix;
  const int64_t first = static_cast<int64_t>(p) << ix.part_shift;
  const int64_t rows = std::max<int64_t>(0, std::min<int64_t>(hi.num_points - first, int64_t(1) << ix.part_shift));
  h->ppresent[p] = true;
  if (rows == 0) return GANN_OK;
  const int64_t vs = ix.vec_stride;
  const int32_t as = ix.adj_stride;
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->pvecs[p]), static_cast<size_t>(rows) * vs));
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->padj[p]), static_cast<size_t>(rows) * as * 4));
  h->device_bytes += rows * (vs + 4 * as);
  const int64_t blk = 1 << 20;
  std::vector<uint8_t> sv(static_cast<size_t>(std::min(blk, rows)) * vs);
  std::vector<uint32_t> sa(static_cast<size_t>(std::min(blk, rows)) * as);
  std::string msg;
  for (int64_t r = 0; r < rows; r += blk) {
    const int64_t c = std::min(blk, rows - r);
    int rc = gann::relayout_records(cfg->index_file, hi, first + r, c, sv.data(), vs, sa.data(), as, msg);
    if (rc) return set_error(rc, msg);
    GANN_CUDA(cudaMemcpy(h->pvecs[p] + r * vs, sv.data(), static_cast<size_t>(c) * vs, cudaMemcpyHostToDevice));
    GANN_CUDA(cudaMemcpy(h->padj[p] + r * as, sa.data(), static_cast<size_t>(c) * as * 4, cudaMemcpyHostToDevice));
  }
  if (with_ncodes) {
    const size_t bytes = static_cast<size_t>(rows) * as * ix.code_stride;
    GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->pncodes[p]), bytes));
    h->device_bytes += static_cast<int64_t>(bytes);
    GANN_CUDA(gann::launch_gather_neighbour_codes(h->padj[p], as, ix.degree, ix.codes, ix.code_stride, rows,
                                                  h->pncodes[p], h->stream));
    GANN_CUDA(cudaStreamSynchronize(h->stream));
  }
  ix.part_vecs[p] = h->pvecs[p];
  ix.part_adj[p] = h->padj[p];
  ix.part_ncodes[p] = h->pncodes[p];
  return GANN_OK;
}

int load_parts(gann_handle* h, const gann_config* cfg) {
  HostIndex& hi = h->hi;
  DeviceIndex& ix = h->ix;
  int shift = 0;
  while ((static_cast<int64_t>(h->part_count) << shift) < hi.num_points) ++shift;
  ix.nparts = h->part_count;
  ix.part_shift = shift;
  ix.local_part = h->part_index;
  ix.vec_stride = gann::round_up(hi.dim, 32) * hi.elem;
  ix.adj_stride = static_cast<int32_t>(gann::round_up(hi.max_m0, 4));
  // neighbour codes per range, on the same rule as the single layout,
  // applied to the ranges this device holds
  const int nown = h->part_index < 0 ? h->part_count : 1;
  const size_t bytes = (static_cast<size_t>(nown) << shift) * ix.adj_stride * ix.code_stride;
  size_t free_b = 0, total_b = 0;
  GANN_CUDA(cudaMemGetInfo(&free_b, &total_b));
  const bool fits = bytes <= total_b / 4 && bytes + (size_t(1) << 30) < free_b;
  if (cfg->layout == 2 && !fits)
    return set_error(GANN_ENOMEM, "gann_open: the neighbour-code copy does not fit in device memory");
  const bool with_ncodes = cfg->layout != 1 && fits;
  h->part_ncodes = with_ncodes ? 1 : 0;
  for (int p = 0; p < h->part_count; ++p) {
    if (h->part_index >= 0 && p != h->part_index) continue;
    int rc = load_part(h, cfg, p, with_ncodes);
    if (rc) return rc;
  }
  if (with_ncodes) {
    // any non-null pointer marks the layout; rows are addressed per range
    for (int p = 0; p < h->part_count && !h->ncodes_on; ++p) h->ncodes_on = h->pncodes[p];
    if (!h->ncodes_on) h->ncodes_on = reinterpret_cast<const uint8_t*>(ix.codes);
    ix.ncodes = h->ncodes_on;
  }
  return GANN_OK;
}

int upload_pivot_table(gann_handle* h) {
  std::vector<float> tab;
  const int w = gann::make_pivot_table(h->hi.pivots_t, h->hi.chunk_offsets, static_cast<int>(h->hi.dim), tab);
  if (w > 0) {
    int rc = dev_upload(h->piv4, tab.data(), tab.size(), h->device_bytes);
    if (rc) return rc;
    h->ix.piv4 = reinterpret_cast<const float4*>(h->piv4);
  }
  h->ix.piv_width = w;
  return GANN_OK;
}

int open_impl(const gann_config* cfg, gann_handle* h) {
  if (!cfg || !cfg->index_file || !cfg->pq_file_prefix)
    return set_error(GANN_EINVAL, "gann_open: index_file and pq_file_prefix are required");
  if (cfg->dtype != GANN_UINT8 && cfg->dtype != GANN_FLOAT)
    return set_error(GANN_EINVAL, "gann_open: dtype must be GANN_UINT8 or GANN_FLOAT");
  h->device = cfg->device;
  h->dtype = cfg->dtype;
  if (cfg->use_gpu_mem < 0 || cfg->use_gpu_mem > 2) return set_error(GANN_EINVAL, "gann_open: use_gpu_mem must be 0, 1 or 2");
  h->host_records = cfg->use_gpu_mem == 0;
  h->storage_records = cfg->use_gpu_mem == 2;
  if (cfg->layout < 0 || cfg->layout > 2) return set_error(GANN_EINVAL, "gann_open: layout must be 0, 1 or 2");
  if (cfg->metric != GANN_METRIC_L2 && cfg->metric != GANN_METRIC_IP)
    return set_error(GANN_EINVAL, "gann_open: metric must be GANN_METRIC_L2 or GANN_METRIC_IP");
  if (cfg->part_count < 0 || cfg->part_count > gann::kMaxParts)
    return set_error(GANN_EINVAL, "gann_open: part_count must be 0..8");
  h->part_count = cfg->part_count > 1 ? cfg->part_count : 0;
  h->part_index = h->part_count ? cfg->part_index : 0;
  if (h->part_count && (h->part_index < -1 || h->part_index >= h->part_count))
    return set_error(GANN_EINVAL, "gann_open: part_index must be -1..part_count-1");
  if (h->part_count && (h->host_records || h->storage_records))
    return set_error(GANN_EUNSUPPORTED, "gann_open: split records need use_gpu_mem = 1");

  // parse and validate every file before touching the GPU
  HostIndex& hi = h->hi;
  hi.dtype = cfg->dtype;
  const int elem = cfg->dtype == GANN_UINT8 ? 1 : 4;
  std::string msg;
  int rc = gann::load_disk_header(cfg->index_file, elem, hi, msg);
  if (rc) return set_error(rc, msg);
  std::vector<uint8_t> codes;
  int64_t rows = 0;
  rc = gann::load_pq(cfg->pq_file_prefix, hi, codes, rows, msg);
  if (rc) return set_error(rc, msg);
  if (cfg->nav_graph_prefix && cfg->nav_graph_prefix[0]) {
    rc = gann::load_nav(cfg->nav_graph_prefix, hi, msg);
    if (rc) return set_error(rc, msg);
  }

  int ndev = 0;
  GANN_CUDA(cudaGetDeviceCount(&ndev));
  if (cfg->device < 0 || cfg->device >= ndev) return set_error(GANN_EINVAL, "gann_open: no such CUDA device");
  GANN_CUDA(cudaSetDevice(h->device));
  h->cuda_ready = true;
  GANN_CUDA(cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, h->device));
  GANN_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  GANN_CUDA(cudaEventCreate(&h->ev0));
  GANN_CUDA(cudaEventCreate(&h->ev1));

  DeviceIndex& ix = h->ix;
  ix.metric = cfg->metric;
  ix.n = hi.num_points;
  ix.dim = static_cast<int32_t>(hi.dim);
  ix.degree = static_cast<int32_t>(hi.max_m0);
  ix.chunks = hi.num_chunks;
  ix.code_stride = static_cast<int32_t>(gann::round_up(hi.num_chunks, 16));
  ix.medoid = hi.medoid;
  if ((rc = dev_upload(h->codes, codes.data(), codes.size(), h->device_bytes))) return rc;
  codes.clear();
  codes.shrink_to_fit();
  if ((rc = dev_upload(h->pivots_t, hi.pivots_t.data(), hi.pivots_t.size(), h->device_bytes))) return rc;
  if ((rc = dev_upload(h->centroid, hi.centroid.data(), hi.centroid.size(), h->device_bytes))) return rc;
  if ((rc = dev_upload(h->chunk_off, hi.chunk_offsets.data(), hi.chunk_offsets.size(), h->device_bytes))) return rc;
  ix.codes = h->codes;
  ix.pivots_t = h->pivots_t;
  ix.centroid = h->centroid;
  ix.chunk_off = h->chunk_off;
  if ((rc = upload_pivot_table(h))) return rc;
  if (hi.has_nav) {
    if ((rc = dev_upload(h->nav_vecs, hi.nav_vecs.data(), hi.nav_vecs.size(), h->device_bytes))) return rc;
    if ((rc = dev_upload(h->nav_adj, hi.nav_adj.data(), hi.nav_adj.size(), h->device_bytes))) return rc;
    if ((rc = dev_upload(h->nav_map, hi.nav_map.data(), hi.nav_map.size(), h->device_bytes))) return rc;
    ix.nav_vecs = h->nav_vecs;
    ix.nav_adj = h->nav_adj;
    ix.nav_map = h->nav_map;
    ix.nav_stride = gann::round_up(hi.dim, 32) * hi.elem;
    ix.nav_row = hi.nav_max_m;
    ix.nav_start = hi.nav_start;
    ix.nav_points = hi.nav_points;
    ix.has_nav = 1;
    hi.nav_vecs.clear();
    hi.nav_vecs.shrink_to_fit();
  }
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->counter), 4 * sizeof(int32_t)));
  GANN_CUDA(alloc_vis(h));
  if (h->part_count) return load_parts(h, cfg);
  if (h->storage_records) return GANN_OK;   // pages are read per hop by the caller
  if ((rc = load_records(h, cfg->index_file))) return rc;
  if (cfg->layout != 1) {
    // neighbour codes next to the adjacency: built on the GPU from the records
    // just loaded (in host-record mode the adjacency is read through UVA)
    const size_t bytes = static_cast<size_t>(hi.num_points) * ix.adj_stride * ix.code_stride;
    size_t free_b = 0, total_b = 0;
    GANN_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const bool fits = bytes <= total_b / 4 && bytes + (size_t(1) << 30) < free_b;
    if (cfg->layout == 2 && !fits)
      return set_error(GANN_ENOMEM, "gann_open: the neighbour-code copy does not fit in device memory");
    if (fits) {
      GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->ncodes), bytes));
      h->device_bytes += static_cast<int64_t>(bytes);
      GANN_CUDA(gann::launch_gather_neighbour_codes(ix.adj, ix.adj_stride, ix.degree, ix.codes, ix.code_stride,
                                                    hi.num_points, h->ncodes, h->stream));
      GANN_CUDA(cudaStreamSynchronize(h->stream));
      ix.ncodes = h->ncodes;
      h->ncodes_on = h->ncodes;
    }
  }
  return GANN_OK;
}

int check_search_args(gann_handle* h, int64_t nq, int32_t topk, int32_t ef) {
  if (!h) return set_error(GANN_EINVAL, "search: null handle");
  if (nq < 0 || nq >= (int64_t(1) << 31) - (int64_t(1) << 24))
    return set_error(GANN_EINVAL, "search: query count out of range");
  if (topk < 1 || topk > ef) return set_error(GANN_EINVAL, "search: need 1 <= topk <= ef_search");
  for (int p = 0; p < h->part_count; ++p)
    if (!h->ppresent[p])
      return set_error(GANN_ESTATE, "search: record range " + std::to_string(p) + " is not attached");
  if (h->hi.dim > 1024) return set_error(GANN_EUNSUPPORTED, "search: dimension above 1024");
  if (ef > gann::search_max_ef())
    return set_error(GANN_EUNSUPPORTED, "search: ef_search above " + std::to_string(gann::search_max_ef()));
  int per_sm_smem = 0;
  cudaDeviceGetAttribute(&per_sm_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, h->device);
  if (gann::search_smem_bytes(h->ix, topk, ef) > static_cast<size_t>(per_sm_smem))
    return set_error(GANN_EUNSUPPORTED, "search: per-query working set exceeds shared memory");
  return GANN_OK;
}

gann::SearchArgs make_args(gann_handle* h, const float* q, int64_t nq, int32_t topk, int32_t ef,
                           int32_t* nns, float* dist, int32_t* found, uint32_t* hops, uint32_t* adc) {
  gann::SearchArgs a;
  a.q = q;
  a.nq = nq;
  a.topk = topk;
  a.ef = ef;
  // generous bounds: a best-first search expands about ef..2*ef nodes
  a.max_hops = std::max(1 << 14, 64 * ef);
  a.nav_max_hops = 1 << 20;
  a.nns = nns;
  a.dist = dist;
  a.found = found;
  a.hops = hops;
  a.adc = adc;
  a.qcounter = h->counter;
  a.err = h->counter + 1;
  a.vis = h->vis;
  a.vis_slots = h->vis_slots;
  return a;
}

template <typename T>
int grow(T*& p, int64_t count) {
  if (p) cudaFree(p);
  p = nullptr;
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&p), sizeof(T) * std::max<int64_t>(count, 1)));
  return GANN_OK;
}

int open_device_impl(const gann_device_index* d, gann_handle* h) {
  if (!d || !d->vectors || !d->adjacency || !d->codes || !d->pivots || !d->centroid || !d->chunk_offsets)
    return set_error(GANN_EINVAL, "gann_open_device: null array");
  if (d->dtype != GANN_UINT8 && d->dtype != GANN_FLOAT) return set_error(GANN_EINVAL, "gann_open_device: bad dtype");
  const int elem = d->dtype == GANN_UINT8 ? 1 : 4;
  if (d->num_points <= 0 || d->num_points >= (int64_t(1) << 31) || d->dim <= 0 || d->dim > 1024)
    return set_error(GANN_EINVAL, "gann_open_device: bad size");
  if (d->max_degree < 1 || d->max_degree > 128 || d->adj_stride < d->max_degree)
    return set_error(GANN_EINVAL, "gann_open_device: bad degree / adjacency stride");
  if (d->vec_stride < d->dim * elem || d->vec_stride % 16 || d->code_stride % 16 || d->pq_chunks < 1 ||
      d->pq_chunks > 128 || d->code_stride < d->pq_chunks || d->adj_stride % 4)
    return set_error(GANN_EINVAL, "gann_open_device: bad row strides");
  if (d->medoid < 0 || d->medoid >= d->num_points) return set_error(GANN_EINVAL, "gann_open_device: bad medoid");
  if (d->metric != GANN_METRIC_L2 && d->metric != GANN_METRIC_IP)
    return set_error(GANN_EINVAL, "gann_open_device: bad metric");
  const uint32_t* off = d->chunk_offsets;
  if (off[0] != 0 || off[d->pq_chunks] != static_cast<uint32_t>(d->dim))
    return set_error(GANN_EINVAL, "gann_open_device: chunk offsets must span [0, dim]");
  for (int i = 0; i < d->pq_chunks; ++i)
    if (off[i + 1] <= off[i]) return set_error(GANN_EINVAL, "gann_open_device: chunk offsets must increase");
  h->owns_records = false;
  h->device = d->device;
  h->dtype = d->dtype;
  HostIndex& hi = h->hi;
  hi.dtype = d->dtype;
  hi.elem = elem;
  hi.num_points = d->num_points;
  hi.dim = d->dim;
  hi.medoid = d->medoid;
  hi.max_m0 = d->max_degree;
  hi.data_size = d->dim * elem;
  hi.max_node_len = hi.data_size + 4 * (d->max_degree + 1);
  hi.num_chunks = d->pq_chunks;
  hi.centroid.assign(d->centroid, d->centroid + d->dim);
  hi.chunk_offsets.assign(off, off + d->pq_chunks + 1);
  hi.pivots_t.resize(static_cast<size_t>(d->dim) * gann::kPivots);
  for (int i = 0; i < gann::kPivots; ++i)
    for (int j = 0; j < d->dim; ++j)
      hi.pivots_t[static_cast<size_t>(j) * gann::kPivots + i] = d->pivots[static_cast<size_t>(i) * d->dim + j];
  int ndev = 0;
  GANN_CUDA(cudaGetDeviceCount(&ndev));
  if (d->device < 0 || d->device >= ndev) return set_error(GANN_EINVAL, "gann_open_device: no such CUDA device");
  GANN_CUDA(cudaSetDevice(h->device));
  h->cuda_ready = true;
  GANN_CUDA(cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, h->device));
  GANN_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  GANN_CUDA(cudaEventCreate(&h->ev0));
  GANN_CUDA(cudaEventCreate(&h->ev1));
  int rc;
  if ((rc = dev_upload(h->pivots_t, hi.pivots_t.data(), hi.pivots_t.size(), h->device_bytes))) return rc;
  if ((rc = dev_upload(h->centroid, hi.centroid.data(), hi.centroid.size(), h->device_bytes))) return rc;
  if ((rc = dev_upload(h->chunk_off, hi.chunk_offsets.data(), hi.chunk_offsets.size(), h->device_bytes))) return rc;
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->counter), 4 * sizeof(int32_t)));
  GANN_CUDA(alloc_vis(h));
  DeviceIndex& ix = h->ix;
  ix.vecs = static_cast<const uint8_t*>(d->vectors);
  ix.adj = d->adjacency;
  ix.codes = d->codes;
  ix.pivots_t = h->pivots_t;
  ix.centroid = h->centroid;
  ix.chunk_off = h->chunk_off;
  ix.n = d->num_points;
  ix.dim = d->dim;
  ix.degree = d->max_degree;
  ix.chunks = d->pq_chunks;
  ix.vec_stride = d->vec_stride;
  ix.adj_stride = d->adj_stride;
  ix.code_stride = d->code_stride;
  ix.medoid = d->medoid;
  ix.metric = d->metric;
  ix.has_nav = 0;
  return upload_pivot_table(h);
}

}  // namespace

extern "C" {

int gann_open_device(const gann_device_index* desc, gann_handle** out) {
  if (!out) return set_error(GANN_EINVAL, "gann_open_device: out is NULL");
  *out = nullptr;
  gann_handle* h = new (std::nothrow) gann_handle();
  if (!h) return set_error(GANN_ENOMEM, "gann_open_device: out of host memory");
  int rc;
  try {
    rc = open_device_impl(desc, h);
  } catch (const std::bad_alloc&) {
    rc = set_error(GANN_ENOMEM, "gann_open_device: out of host memory");
  }
  if (rc != GANN_OK) {
    h->release();
    delete h;
    return rc;
  }
  *out = h;
  return GANN_OK;
}

int gann_open(const gann_config* cfg, gann_handle** out) {
  if (!out) return set_error(GANN_EINVAL, "gann_open: out is NULL");
  *out = nullptr;
  gann_handle* h = new (std::nothrow) gann_handle();
  if (!h) return set_error(GANN_ENOMEM, "gann_open: out of host memory");
  int rc;
  try {
    rc = open_impl(cfg, h);
  } catch (const std::bad_alloc&) {
    rc = set_error(GANN_ENOMEM, "gann_open: out of host memory");
  }
  if (rc != GANN_OK) {
    h->release();
    delete h;
    return rc;
  }
  *out = h;
  return GANN_OK;
}

// ----------------------------------------------------------------- host-driven hops
struct gann_hop_batch {
  gann_handle* h = nullptr;
  gann::HopState s;
  float* d_q = nullptr;
  uint8_t* d_pages = nullptr;
  void release() {
    if (!h) return;
    cudaSetDevice(h->device);
    for (void* p : {static_cast<void*>(s.qpp), static_cast<void*>(s.lut), static_cast<void*>(s.pool),
                    static_cast<void*>(s.psize), static_cast<void*>(s.request), static_cast<void*>(s.nns),
                    static_cast<void*>(s.dist), static_cast<void*>(s.found), static_cast<void*>(s.hops),
                    static_cast<void*>(s.err), static_cast<void*>(d_q), static_cast<void*>(d_pages)})
      if (p) cudaFree(p);
    s = gann::HopState();
    d_q = nullptr;
    d_pages = nullptr;
  }
};

}  // extern "C"

namespace {
template <typename T>
cudaError_t dalloc(T*& p, int64_t count) {
  return cudaMalloc(reinterpret_cast<void**>(&p), sizeof(T) * static_cast<size_t>(std::max<int64_t>(count, 1)));
}

int hop_begin_impl(gann_handle* h, const float* queries, int64_t nq, int32_t topk, int32_t ef, gann_hop_batch* b) {
  const HostIndex& hi = h->hi;
  gann::HopState& s = b->s;
  s.nq = nq;
  s.topk = topk;
  s.ef = ef;
  s.max_hops = std::max(1 << 14, 64 * ef);
  s.nav_max_hops = 1 << 20;
  GANN_CUDA(cudaSetDevice(h->device));
  GANN_CUDA(dalloc(s.qpp, nq * hi.dim));
  GANN_CUDA(dalloc(s.lut, nq * hi.num_chunks * gann::kPivots));
  GANN_CUDA(dalloc(s.pool, nq * ef));
  GANN_CUDA(dalloc(s.psize, nq));
  GANN_CUDA(dalloc(s.request, nq));
  GANN_CUDA(dalloc(s.nns, nq * topk));
  GANN_CUDA(dalloc(s.dist, nq * topk));
  GANN_CUDA(dalloc(s.found, nq));
  GANN_CUDA(dalloc(s.hops, nq));
  GANN_CUDA(dalloc(s.err, 3));
  GANN_CUDA(dalloc(b->d_q, nq * hi.dim));
  GANN_CUDA(dalloc(b->d_pages, nq * gann::kPageSize));
  GANN_CUDA(cudaMemsetAsync(s.err, 0, 3 * sizeof(int32_t), h->stream));
  if (nq > 0)
    GANN_CUDA(cudaMemcpyAsync(b->d_q, queries, sizeof(float) * nq * hi.dim, cudaMemcpyHostToDevice, h->stream));
  GANN_CUDA(gann::launch_hop_begin(h->ix, b->d_q, s, h->dtype, h->stream));
  GANN_CUDA(cudaStreamSynchronize(h->stream));
  return GANN_OK;
}
}  // namespace

extern "C" {

int gann_hop_begin(gann_handle* h, const float* queries, int64_t nq, int32_t topk, int32_t ef_search,
                   gann_hop_batch** out) {
  if (!out) return set_error(GANN_EINVAL, "gann_hop_begin: null output");
  *out = nullptr;
  int rc = check_search_args(h, nq, topk, ef_search);
  if (rc) return rc;
  if (nq > 0 && !queries) return set_error(GANN_EINVAL, "gann_hop_begin: null queries");
  if (h->part_count) return set_error(GANN_EUNSUPPORTED, "gann_hop_begin: not with split records");
  if ((h->hi.dim * h->hi.elem) % 4 != 0 || h->hi.max_node_len % 4 != 0)
    return set_error(GANN_EUNSUPPORTED, "gann_hop_begin: records must be 4-byte aligned within a page");
  auto* b = new (std::nothrow) gann_hop_batch;
  if (!b) return set_error(GANN_ENOMEM, "gann_hop_begin: out of host memory");
  b->h = h;
  rc = hop_begin_impl(h, queries, nq, topk, ef_search, b);
  if (rc) {
    b->release();
    delete b;
    return rc;
  }
  *out = b;
  return GANN_OK;
}

int gann_hop_requests(gann_hop_batch* b, int32_t* node_ids, int64_t* active) {
  if (!b || !b->h || (b->s.nq > 0 && !node_ids)) return set_error(GANN_EINVAL, "gann_hop_requests: bad argument");
  gann_handle* h = b->h;
  GANN_CUDA(cudaSetDevice(h->device));
  if (b->s.nq > 0) {
    GANN_CUDA(cudaMemcpyAsync(node_ids, b->s.request, sizeof(int32_t) * b->s.nq, cudaMemcpyDeviceToHost, h->stream));
    GANN_CUDA(cudaStreamSynchronize(h->stream));
  }
  int64_t n = 0;
  for (int64_t i = 0; i < b->s.nq; ++i) n += node_ids[i] >= 0;
  if (active) *active = n;
  return GANN_OK;
}

int gann_hop_step(gann_hop_batch* b, const void* pages) {
  if (!b || !b->h || (b->s.nq > 0 && !pages)) return set_error(GANN_EINVAL, "gann_hop_step: bad argument");
  gann_handle* h = b->h;
  GANN_CUDA(cudaSetDevice(h->device));
  if (b->s.nq == 0) return GANN_OK;
  GANN_CUDA(cudaMemcpyAsync(b->d_pages, pages, static_cast<size_t>(b->s.nq) * gann::kPageSize,
                            cudaMemcpyHostToDevice, h->stream));
  GANN_CUDA(gann::launch_hop_step(h->ix, b->s, b->d_pages, static_cast<int32_t>(h->hi.max_node_len),
                                  static_cast<int32_t>(h->hi.nodes_per_page), h->dtype, h->stream));
  GANN_CUDA(cudaStreamSynchronize(h->stream));
  return GANN_OK;
}

int gann_hop_finish(gann_hop_batch* b, int32_t* nns, float* distances, int32_t* found_cnt) {
  if (!b || !b->h || (b->s.nq > 0 && (!nns || !distances || !found_cnt)))
    return set_error(GANN_EINVAL, "gann_hop_finish: bad argument");
  gann_handle* h = b->h;
  const gann::HopState& s = b->s;
  GANN_CUDA(cudaSetDevice(h->device));
  if (s.nq > 0) {
    GANN_CUDA(cudaMemcpyAsync(nns, s.nns, sizeof(int32_t) * s.nq * s.topk, cudaMemcpyDeviceToHost, h->stream));
    GANN_CUDA(cudaMemcpyAsync(distances, s.dist, sizeof(float) * s.nq * s.topk, cudaMemcpyDeviceToHost, h->stream));
    GANN_CUDA(cudaMemcpyAsync(found_cnt, s.found, sizeof(int32_t) * s.nq, cudaMemcpyDeviceToHost, h->stream));
  }
  int32_t errs[3] = {0, 0, 0};
  GANN_CUDA(cudaMemcpyAsync(errs, s.err, sizeof(errs), cudaMemcpyDeviceToHost, h->stream));
  GANN_CUDA(cudaStreamSynchronize(h->stream));
  if (errs[2]) return set_error(GANN_EINVAL, "gann_hop_finish: " + std::to_string(errs[2]) +
                                                 " page(s) held records that are not this index's");
  return GANN_OK;
}

int gann_read_pages(const char* index_file, const int32_t* node_ids, int64_t n, int32_t nodes_per_page,
                    void* pages, int32_t threads) {
  if (!index_file || n < 0 || nodes_per_page <= 0 || (n > 0 && (!node_ids || !pages)))
    return set_error(GANN_EINVAL, "gann_read_pages: bad argument");
  const int fd = ::open(index_file, O_RDONLY);
  if (fd < 0) return set_error(GANN_EIO, std::string("gann_read_pages: cannot open ") + index_file);
  int nt = threads > 0 ? threads : static_cast<int>(std::thread::hardware_concurrency());
  nt = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({static_cast<int64_t>(nt), int64_t(64), n})));
  std::atomic<int64_t> bad{-1};
  auto work = [&](int t) {
    for (int64_t i = t; i < n; i += nt) {
      const int32_t id = node_ids[i];
      if (id < 0) continue;
      const off_t off = static_cast<off_t>(gann::kPageSize) * (1 + id / nodes_per_page);
      uint8_t* dst = static_cast<uint8_t*>(pages) + i * gann::kPageSize;
      ssize_t got = 0;
      while (got < gann::kPageSize) {
        const ssize_t r = ::pread(fd, dst + got, gann::kPageSize - got, off + got);
        if (r <= 0) break;
        got += r;
      }
      if (got != gann::kPageSize) bad.store(i);
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; ++t) pool.emplace_back(work, t);
  work(0);
  for (auto& th : pool) th.join();
  ::close(fd);
  if (bad.load() >= 0)
    return set_error(GANN_EIO, "gann_read_pages: short read for node " + std::to_string(node_ids[bad.load()]));
  return GANN_OK;
}

int gann_hop_free(gann_hop_batch* b) {
  if (!b) return GANN_OK;
  b->release();
  delete b;
  return GANN_OK;
}

int gann_close(gann_handle* h) {
  if (!h) return GANN_OK;
  h->release();
  delete h;
  return GANN_OK;
}

const char* gann_last_error(void) { return g_last_error.c_str(); }

namespace {
// Content of a gann_part_export blob.
struct PartBlob {
  uint32_t magic, version;
  int32_t part, part_count, part_shift, has_ncodes;
  int64_t num_points, rows, vec_stride;
  int32_t adj_stride, code_stride;
  cudaIpcMemHandle_t vecs, adj, ncodes;
};
constexpr uint32_t kBlobMagic = 0x47414e50u;  // "GANP"
static_assert(sizeof(PartBlob) <= GANN_PART_BLOB_BYTES, "blob too large");

int64_t part_rows(const gann_handle* h, int p) {
  const int64_t first = static_cast<int64_t>(p) << h->ix.part_shift;
  return std::max<int64_t>(0, std::min<int64_t>(h->hi.num_points - first, int64_t(1) << h->ix.part_shift));
}
}  // namespace

int gann_part_export(gann_handle* h, void* blob, int64_t blob_bytes) {
  if (!h || !blob || blob_bytes < GANN_PART_BLOB_BYTES) return set_error(GANN_EINVAL, "gann_part_export: bad argument");
  if (h->part_count < 2 || h->part_index < 0)
    return set_error(GANN_ESTATE, "gann_part_export: the handle does not own one record range");
  const int p = h->part_index;
  PartBlob b;
  std::memset(&b, 0, sizeof(b));
  b.magic = kBlobMagic;
  b.version = GANN_ABI_VERSION;
  b.part = p;
  b.part_count = h->part_count;
  b.part_shift = h->ix.part_shift;
  b.has_ncodes = h->part_ncodes;
  b.num_points = h->hi.num_points;
  b.rows = part_rows(h, p);
  b.vec_stride = h->ix.vec_stride;
  b.adj_stride = h->ix.adj_stride;
  b.code_stride = h->ix.code_stride;
  GANN_CUDA(cudaSetDevice(h->device));
  if (b.rows > 0) {
    GANN_CUDA(cudaIpcGetMemHandle(&b.vecs, h->pvecs[p]));
    GANN_CUDA(cudaIpcGetMemHandle(&b.adj, h->padj[p]));
    if (h->pncodes[p]) GANN_CUDA(cudaIpcGetMemHandle(&b.ncodes, h->pncodes[p]));
  }
  std::memset(blob, 0, GANN_PART_BLOB_BYTES);
  std::memcpy(blob, &b, sizeof(b));
  return GANN_OK;
}

int gann_part_attach(gann_handle* h, int32_t part, const void* blob, int64_t blob_bytes) {
  if (!h || !blob || blob_bytes < GANN_PART_BLOB_BYTES) return set_error(GANN_EINVAL, "gann_part_attach: bad argument");
  PartBlob b;
  std::memcpy(&b, blob, sizeof(b));
  if (b.magic != kBlobMagic || b.version != GANN_ABI_VERSION)
    return set_error(GANN_EINVAL, "gann_part_attach: not a record-range blob of this library");
  if (h->part_count < 2 || part < 0 || part >= h->part_count || b.part != part)
    return set_error(GANN_EINVAL, "gann_part_attach: range index out of range or not the blob's range");
  if (h->ppresent[part]) return set_error(GANN_ESTATE, "gann_part_attach: the range is already present");
  if (b.part_count != h->part_count || b.part_shift != h->ix.part_shift || b.num_points != h->hi.num_points ||
      b.rows != part_rows(h, part) || b.vec_stride != h->ix.vec_stride || b.adj_stride != h->ix.adj_stride ||
      b.code_stride != h->ix.code_stride || b.has_ncodes != h->part_ncodes)
    return set_error(GANN_EINVAL, "gann_part_attach: the range was exported from a different index or layout");
  GANN_CUDA(cudaSetDevice(h->device));
  h->pattached[part] = true;
  if (b.rows > 0) {
    void* v = nullptr;
    void* a = nullptr;
    void* c = nullptr;
    GANN_CUDA(cudaIpcOpenMemHandle(&v, b.vecs, cudaIpcMemLazyEnablePeerAccess));
    h->pvecs[part] = static_cast<uint8_t*>(v);
    GANN_CUDA(cudaIpcOpenMemHandle(&a, b.adj, cudaIpcMemLazyEnablePeerAccess));
    h->padj[part] = static_cast<uint32_t*>(a);
    if (b.has_ncodes) {
      GANN_CUDA(cudaIpcOpenMemHandle(&c, b.ncodes, cudaIpcMemLazyEnablePeerAccess));
      h->pncodes[part] = static_cast<uint8_t*>(c);
    }
  }
  h->ix.part_vecs[part] = h->pvecs[part];
  h->ix.part_adj[part] = h->padj[part];
  h->ix.part_ncodes[part] = h->pncodes[part];
  h->ppresent[part] = true;
  return GANN_OK;
}

int gann_set_option(gann_handle* h, int32_t option, int64_t value) {
  if (!h) return set_error(GANN_EINVAL, "gann_set_option: null handle");
  switch (option) {
    case GANN_OPT_ADC_MODE:
      if (value < 0 || value > 3) return set_error(GANN_EINVAL, "gann_set_option: ADC mode must be 0, 1, 2 or 3");
      if (value == 2 && (h->ix.piv_width == 0 || h->ix.dim > 128))
        return set_error(GANN_EUNSUPPORTED, "gann_set_option: pivot mode needs <= 4 dims per chunk and dim <= 128");
      if (value == 3 && (h->ix.piv_width == 0 || h->ix.dim > 128 || h->ix.chunks > 32 ||
                         h->ix.metric != GANN_METRIC_L2))
        return set_error(GANN_EUNSUPPORTED,
                         "gann_set_option: filtered mode needs L2, <= 4 dims per chunk, <= 32 chunks and dim <= 128");
      h->ix.adc_mode = static_cast<int32_t>(value);
      return GANN_OK;
    case GANN_OPT_PIVOT_WARPS:
      if (value != 0 && (value < 8 || value > 24))
        return set_error(GANN_EINVAL, "gann_set_option: pivot warps must be 0 or 8..24");
      h->ix.piv_warps = static_cast<int32_t>(value);
      return GANN_OK;
    case GANN_OPT_NEIGHBOUR_CODES:
      if (value != 0 && value != 1) return set_error(GANN_EINVAL, "gann_set_option: neighbour codes must be 0 or 1");
      if (value == 1 && !h->ncodes_on)
        return set_error(GANN_ESTATE, "gann_set_option: the handle was opened without the neighbour-code copy");
      h->ix.ncodes = value ? h->ncodes_on : nullptr;
      return GANN_OK;
    default:
      return set_error(GANN_EINVAL, "gann_set_option: unknown option");
  }
}

int gann_index_info(const gann_handle* h, gann_info* out) {
  if (!h || !out) return set_error(GANN_EINVAL, "gann_index_info: null argument");
  std::memset(out, 0, sizeof(*out));
  out->num_points = h->hi.num_points;
  out->dim = static_cast<int32_t>(h->hi.dim);
  out->max_degree = static_cast<int32_t>(h->hi.max_m0);
  out->pq_chunks = h->hi.num_chunks;
  out->dtype = h->dtype;
  out->medoid = h->hi.medoid;
  out->node_len = static_cast<int32_t>(h->hi.max_node_len);
  out->nodes_per_page = static_cast<int32_t>(h->hi.nodes_per_page);
  out->nav_points = static_cast<int32_t>(h->hi.nav_points);
  out->nav_start = h->hi.nav_start;
  out->device_bytes = h->device_bytes;
  return GANN_OK;
}

int gann_search_device(gann_handle* h, const float* d_queries, int64_t nq, int32_t topk, int32_t ef_search,
                       int32_t* d_nns, float* d_distances, int32_t* d_found_cnt, uint32_t* d_hops_out,
                       void* stream) {
  int rc = check_search_args(h, nq, topk, ef_search);
  if (rc) return rc;
  if (h->storage_records) return set_error(GANN_ESTATE, "search: records are on storage; use gann_hop_*");
  if (nq == 0) return GANN_OK;
  if (!d_queries || !d_nns || !d_distances || !d_found_cnt)
    return set_error(GANN_EINVAL, "gann_search_device: null buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GANN_CUDA(cudaSetDevice(h->device));
  GANN_CUDA(cudaMemsetAsync(h->counter, 0, 4 * sizeof(int32_t), st));
  gann::SearchArgs a = make_args(h, d_queries, nq, topk, ef_search, d_nns, d_distances, d_found_cnt,
                                 d_hops_out, nullptr);
  GANN_CUDA(gann::launch_search(h->ix, a, h->dtype, h->sm_count, st));
  return GANN_OK;
}

int gann_search(gann_handle* h, const float* queries, int64_t nq, int32_t topk, int32_t ef_search,
                int32_t* nns, float* distances, int32_t* found_cnt, gann_stats* stats) {
  const auto t0 = std::chrono::steady_clock::now();
  int rc = check_search_args(h, nq, topk, ef_search);
  if (rc) return rc;
  if (h->storage_records) return set_error(GANN_ESTATE, "search: records are on storage; use gann_hop_*");
  if (stats) std::memset(stats, 0, sizeof(*stats));
  if (nq == 0) return GANN_OK;
  if (!queries || !nns || !distances || !found_cnt) return set_error(GANN_EINVAL, "gann_search: null buffer");
  GANN_CUDA(cudaSetDevice(h->device));
  const int64_t dim = h->hi.dim;
  if (nq * dim > h->cap_q) {
    if ((rc = grow(h->d_q, nq * dim))) return rc;
    h->cap_q = nq * dim;
  }
  if (nq * topk > h->cap_out || nq > h->cap_out) {
    const int64_t c = std::max(nq * topk, nq);
    if ((rc = grow(h->d_nns, c)) || (rc = grow(h->d_dist, c)) || (rc = grow(h->d_found, c)) ||
        (rc = grow(h->d_hops, c)) || (rc = grow(h->d_adc, c)))
      return rc;
    h->cap_out = c;
  }
  cudaStream_t st = h->stream;
  GANN_CUDA(cudaMemcpyAsync(h->d_q, queries, sizeof(float) * nq * dim, cudaMemcpyHostToDevice, st));
  GANN_CUDA(cudaMemsetAsync(h->counter, 0, 4 * sizeof(int32_t), st));
  gann::SearchArgs a = make_args(h, h->d_q, nq, topk, ef_search, h->d_nns, h->d_dist, h->d_found, h->d_hops,
                                 h->d_adc);
  GANN_CUDA(cudaEventRecord(h->ev0, st));
  GANN_CUDA(gann::launch_search(h->ix, a, h->dtype, h->sm_count, st));
  GANN_CUDA(cudaEventRecord(h->ev1, st));
  GANN_CUDA(cudaMemcpyAsync(nns, h->d_nns, sizeof(int32_t) * nq * topk, cudaMemcpyDeviceToHost, st));
  GANN_CUDA(cudaMemcpyAsync(distances, h->d_dist, sizeof(float) * nq * topk, cudaMemcpyDeviceToHost, st));
  GANN_CUDA(cudaMemcpyAsync(found_cnt, h->d_found, sizeof(int32_t) * nq, cudaMemcpyDeviceToHost, st));
  std::vector<uint32_t> hops, adc;
  int32_t errs[4] = {0, 0, 0, 0};
  if (stats) {
    hops.resize(nq);
    adc.resize(nq);
    GANN_CUDA(cudaMemcpyAsync(hops.data(), h->d_hops, sizeof(uint32_t) * nq, cudaMemcpyDeviceToHost, st));
    GANN_CUDA(cudaMemcpyAsync(adc.data(), h->d_adc, sizeof(uint32_t) * nq, cudaMemcpyDeviceToHost, st));
    GANN_CUDA(cudaMemcpyAsync(errs, h->counter, sizeof(errs), cudaMemcpyDeviceToHost, st));
  }
  GANN_CUDA(cudaStreamSynchronize(st));
  if (stats) {
    float ms = 0.f;
    GANN_CUDA(cudaEventElapsedTime(&ms, h->ev0, h->ev1));
    stats->run_time = ms * 1e-3;
    int64_t sh = 0, sa = 0;
    for (int64_t i = 0; i < nq; ++i) {
      sh += hops[i];
      sa += adc[i];
    }
    stats->hops = sh;
    stats->adc_evals = sa;
    stats->capped_queries = errs[1];
    // algorithmic bytes: query + per hop one record + one PQ code row per
    // evaluated neighbour + the top-k written back
    stats->bytes_touched = nq * dim * h->hi.elem + sh * h->hi.max_node_len + sa * h->hi.num_chunks +
                           nq * topk * 8;
    stats->total_time = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
  return GANN_OK;
}

int gann_probe_lut(gann_handle* h, const float* queries, int64_t nq, float* luts) {
  if (!h || nq < 0 || (nq > 0 && (!queries || !luts))) return set_error(GANN_EINVAL, "gann_probe_lut: bad argument");
  if (nq == 0) return GANN_OK;
  GANN_CUDA(cudaSetDevice(h->device));
  float *dq = nullptr, *dl = nullptr;
  const size_t lut_n = static_cast<size_t>(nq) * h->hi.num_chunks * gann::kPivots;
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&dq), sizeof(float) * nq * h->hi.dim));
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&dl), sizeof(float) * lut_n);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dq, queries, sizeof(float) * nq * h->hi.dim, cudaMemcpyHostToDevice, h->stream);
  if (e == cudaSuccess) e = gann::launch_probe_lut(h->ix, dq, nq, dl, h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(luts, dl, sizeof(float) * lut_n, cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  cudaFree(dq);
  cudaFree(dl);
  if (e != cudaSuccess) return set_error(GANN_ECUDA, std::string("gann_probe_lut: ") + cudaGetErrorString(e));
  return GANN_OK;
}

int gann_probe_entry(gann_handle* h, const float* queries, int64_t nq, int32_t* sample_idx, int32_t* entry_ids) {
  if (!h || nq < 0 || (nq > 0 && (!queries || !sample_idx || !entry_ids)))
    return set_error(GANN_EINVAL, "gann_probe_entry: bad argument");
  if (!h->ix.has_nav) return set_error(GANN_ESTATE, "gann_probe_entry: index opened without a nav graph");
  if (nq == 0) return GANN_OK;
  GANN_CUDA(cudaSetDevice(h->device));
  float* dq = nullptr;
  int32_t* dbuf = nullptr;
  GANN_CUDA(cudaMalloc(reinterpret_cast<void**>(&dq), sizeof(float) * nq * h->hi.dim));
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&dbuf), sizeof(int32_t) * (2 * nq + 1));
  if (e == cudaSuccess) e = cudaMemsetAsync(dbuf, 0, sizeof(int32_t) * (2 * nq + 1), h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dq, queries, sizeof(float) * nq * h->hi.dim, cudaMemcpyHostToDevice, h->stream);
  if (e == cudaSuccess) e = gann::launch_probe_entry(h->ix, dq, nq, h->dtype, dbuf, dbuf + nq, dbuf + 2 * nq, h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(sample_idx, dbuf, sizeof(int32_t) * nq, cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(entry_ids, dbuf + nq, sizeof(int32_t) * nq, cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  cudaFree(dq);
  cudaFree(dbuf);
  if (e != cudaSuccess) return set_error(GANN_ECUDA, std::string("gann_probe_entry: ") + cudaGetErrorString(e));
  return GANN_OK;
}

int gann_pivot_sample(int64_t n, int64_t s, uint32_t seed, int32_t* out) {
  if (n <= 0 || n >= (int64_t(1) << 31) || s < 0 || s > n || (s > 0 && !out))
    return set_error(GANN_EINVAL, "gann_pivot_sample: need 0 <= s <= n < 2^31");
  try {
    std::vector<int> v(static_cast<size_t>(n));
    std::iota(v.begin(), v.end(), 0);
    std::mt19937 gen(seed);
    std::shuffle(v.begin(), v.end(), gen);
    v.resize(static_cast<size_t>(s));
    std::sort(v.begin(), v.end());
    std::copy(v.begin(), v.end(), out);
  } catch (const std::bad_alloc&) {
    return set_error(GANN_ENOMEM, "gann_pivot_sample: out of host memory");
  }
  return GANN_OK;
}

int gann_exact_knn(const void* d_base, int64_t num_points, int64_t base_stride, int32_t dim, int32_t dtype,
                   const void* d_queries, int64_t query_stride, int64_t nq, int32_t k, int32_t metric,
                   int32_t* d_ids, float* d_distances, int32_t device, void* stream) {
  if (dtype != GANN_UINT8 && dtype != GANN_FLOAT) return set_error(GANN_EINVAL, "gann_exact_knn: bad dtype");
  if (metric != GANN_METRIC_L2 && metric != GANN_METRIC_IP) return set_error(GANN_EINVAL, "gann_exact_knn: bad metric");
  const int64_t elem = dtype == GANN_UINT8 ? 1 : 4;
  if (num_points <= 0 || num_points >= (int64_t(1) << 31) || dim <= 0 || dim > 4096 || nq < 0)
    return set_error(GANN_EINVAL, "gann_exact_knn: bad size");
  if (k < 1 || k > gann::exact_knn_max_k() || k > num_points)
    return set_error(GANN_EINVAL, "gann_exact_knn: need 1 <= k <= min(128, num_points)");
  if (base_stride < dim * elem || query_stride < dim * elem || base_stride % 16 || query_stride % 16)
    return set_error(GANN_EINVAL, "gann_exact_knn: strides must cover a row and be multiples of 16 bytes");
  if (nq == 0) return GANN_OK;
  if (!d_base || !d_queries || !d_ids || !d_distances || reinterpret_cast<uintptr_t>(d_base) % 16 ||
      reinterpret_cast<uintptr_t>(d_queries) % 16)
    return set_error(GANN_EINVAL, "gann_exact_knn: null or unaligned buffer");
  int ndev = 0;
  GANN_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_error(GANN_EINVAL, "gann_exact_knn: no such CUDA device");
  int prev = 0;
  GANN_CUDA(cudaGetDevice(&prev));
  GANN_CUDA(cudaSetDevice(device));
  int sm = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess)
    e = gann::launch_exact_knn(d_base, num_points, base_stride, dim, dtype, d_queries, query_stride, nq, k, metric,
                               d_ids, d_distances, sm, static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  if (e != cudaSuccess)
    return set_error(e == cudaErrorMemoryAllocation ? GANN_ENOMEM : GANN_ECUDA,
                     std::string("gann_exact_knn: ") + cudaGetErrorString(e));
  return GANN_OK;
}

int gann_robust_prune(const void* d_vectors, int64_t num_points, int64_t stride, int32_t dim, int32_t dtype,
                      const int32_t* d_points, int64_t count, const int32_t* d_cand, const float* d_cand_dist,
                      int32_t k, int32_t r, float alpha, int32_t* d_out, float* d_out_dist, int32_t device,
                      void* stream) {
  if (dtype != GANN_UINT8 && dtype != GANN_FLOAT) return set_error(GANN_EINVAL, "gann_robust_prune: bad dtype");
  const int64_t elem = dtype == GANN_UINT8 ? 1 : 4;
  if (num_points <= 0 || num_points >= (int64_t(1) << 31) || dim <= 0 || dim > 4096 || count < 0)
    return set_error(GANN_EINVAL, "gann_robust_prune: bad size");
  if (k < 1 || k > gann::prune_max_candidates() || r < 1 || !(alpha >= 1.f))
    return set_error(GANN_EINVAL, "gann_robust_prune: need 1 <= k <= 256, r >= 1, alpha >= 1");
  if (stride < dim * elem || stride % 16 || reinterpret_cast<uintptr_t>(d_vectors) % 16)
    return set_error(GANN_EINVAL, "gann_robust_prune: vector rows must be 16-byte aligned");
  if (count == 0) return GANN_OK;
  if (!d_vectors || !d_points || !d_cand || !d_cand_dist || !d_out || !d_out_dist)
    return set_error(GANN_EINVAL, "gann_robust_prune: null buffer");
  int ndev = 0;
  GANN_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_error(GANN_EINVAL, "gann_robust_prune: no such CUDA device");
  int prev = 0;
  GANN_CUDA(cudaGetDevice(&prev));
  GANN_CUDA(cudaSetDevice(device));
  int sm = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess)
    e = gann::launch_robust_prune(d_vectors, num_points, stride, dim, dtype, d_points, count, d_cand, d_cand_dist,
                                  k, r, alpha, d_out, d_out_dist, sm, static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return set_error(GANN_ECUDA, std::string("gann_robust_prune: ") + cudaGetErrorString(e));
  return GANN_OK;
}

int gann_sort_unique_rows(const int32_t* d_ids, const float* d_dists, int64_t rows, int32_t k, int32_t* d_out_ids,
                          float* d_out_dists, int32_t device, void* stream) {
  if (rows < 0 || k < 1 || k > gann::prune_max_candidates())
    return set_error(GANN_EINVAL, "gann_sort_unique_rows: need rows >= 0 and 1 <= k <= 256");
  if (rows == 0) return GANN_OK;
  if (!d_ids || !d_dists || !d_out_ids || !d_out_dists) return set_error(GANN_EINVAL, "gann_sort_unique_rows: null buffer");
  int ndev = 0;
  GANN_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_error(GANN_EINVAL, "gann_sort_unique_rows: no such CUDA device");
  int prev = 0;
  GANN_CUDA(cudaGetDevice(&prev));
  GANN_CUDA(cudaSetDevice(device));
  int sm = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess)
    e = gann::launch_sort_unique_rows(d_ids, d_dists, rows, k, d_out_ids, d_out_dists, sm,
                                      static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return set_error(GANN_ECUDA, std::string("gann_sort_unique_rows: ") + cudaGetErrorString(e));
  return GANN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free search (gann_search_noalloc): every piece of library-side
// device state of a call lives in this one static array, laid out per call as
//   [0, 256)       work counter and error counters (cleared on every call)
//   centroid       dim floats
//   chunk offsets  pq_chunks + 1 int32
//   raw pivots     256 x dim floats, copied from the caller's host array
//   pivots_t       dim x 256 floats (transposed on the GPU)
//   pivot table    pq_chunks x 256 float4 (only when chunks have <= 4 dims and dim <= 128)
// Host code never uses the array's name as an address: the device address
// comes from cudaGetSymbolAddress, looked up once per device.
namespace {

constexpr size_t kNoallocBytes = GANN_NOALLOC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoallocMaxDevices] = {};

__global__ void noalloc_stage_tables(const float* raw, const int32_t* off, int dim, int m, int with_piv,
                                     float* pivots_t, float4* piv4) {
  const int stride = gridDim.x * blockDim.x;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < dim * gann::kPivots; idx += stride) {
    const int d = idx / gann::kPivots, j = idx % gann::kPivots;
    pivots_t[idx] = raw[j * dim + d];
  }
  if (!with_piv) return;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < m * gann::kPivots; idx += stride) {
    const int c = idx / gann::kPivots, j = idx % gann::kPivots;
    const int a0 = off[c], a1 = off[c + 1];
    float r[4];
    for (int t = 0; t < 4; ++t) r[t] = a0 + t < a1 ? raw[j * dim + a0 + t] : 0.f;
    piv4[idx] = make_float4(r[0], r[1], r[2], r[3]);
  }
}

size_t noalloc_align(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

extern "C" int gann_search_noalloc(const gann_device_index* d, const float* d_queries, int64_t nq, int32_t topk,
                                   int32_t ef_search, int32_t* d_nns, float* d_distances, int32_t* d_found_cnt,
                                   void* stream) {
  if (!d || !d->vectors || !d->adjacency || !d->codes || !d->pivots || !d->centroid || !d->chunk_offsets)
    return set_error(GANN_EINVAL, "gann_search_noalloc: null array in the index descriptor");
  if (d->dtype != GANN_UINT8 && d->dtype != GANN_FLOAT) return set_error(GANN_EINVAL, "gann_search_noalloc: bad dtype");
  const int elem = d->dtype == GANN_UINT8 ? 1 : 4;
  if (d->num_points <= 0 || d->num_points >= (int64_t(1) << 31) || d->dim <= 0 || d->dim > 1024)
    return set_error(GANN_EINVAL, "gann_search_noalloc: bad index size");
  if (d->max_degree < 1 || d->max_degree > 128 || d->adj_stride < d->max_degree || d->adj_stride % 4)
    return set_error(GANN_EINVAL, "gann_search_noalloc: bad degree / adjacency stride");
  if (d->vec_stride < d->dim * elem || d->vec_stride % 16 || d->code_stride % 16 || d->pq_chunks < 1 ||
      d->pq_chunks > 128 || d->code_stride < d->pq_chunks)
    return set_error(GANN_EINVAL, "gann_search_noalloc: bad row strides");
  if (d->medoid < 0 || d->medoid >= d->num_points) return set_error(GANN_EINVAL, "gann_search_noalloc: bad medoid");
  if (d->metric != GANN_METRIC_L2 && d->metric != GANN_METRIC_IP)
    return set_error(GANN_EINVAL, "gann_search_noalloc: bad metric");
  const uint32_t* off = d->chunk_offsets;
  const int m = d->pq_chunks, dim = d->dim;
  if (off[0] != 0 || off[m] != static_cast<uint32_t>(dim))
    return set_error(GANN_EINVAL, "gann_search_noalloc: chunk offsets must span [0, dim]");
  int maxw = 0;
  bool all3 = true;
  for (int i = 0; i < m; ++i) {
    if (off[i + 1] <= off[i]) return set_error(GANN_EINVAL, "gann_search_noalloc: chunk offsets must increase");
    maxw = std::max(maxw, static_cast<int>(off[i + 1] - off[i]));
    all3 = all3 && off[i + 1] - off[i] == 3;
  }
  if (nq < 0 || nq >= (int64_t(1) << 31) - (int64_t(1) << 24))
    return set_error(GANN_EINVAL, "gann_search_noalloc: query count out of range");
  if (topk < 1 || topk > ef_search) return set_error(GANN_EINVAL, "gann_search_noalloc: need 1 <= topk <= ef_search");
  if (ef_search > gann::search_max_ef())
    return set_error(GANN_EUNSUPPORTED, "gann_search_noalloc: ef_search above " + std::to_string(gann::search_max_ef()));
  if (nq > 0 && (!d_queries || !d_nns || !d_distances || !d_found_cnt))
    return set_error(GANN_EINVAL, "gann_search_noalloc: null buffer");

  // scratch layout for this index
  const int piv_width = (maxw <= 4 && dim <= 128) ? (all3 ? 3 : 4) : 0;
  size_t o = 256;
  const size_t o_cen = o;
  o = noalloc_align(o + sizeof(float) * dim);
  const size_t o_off = o;
  o = noalloc_align(o + sizeof(int32_t) * (m + 1));
  const size_t o_raw = o;
  o = noalloc_align(o + sizeof(float) * gann::kPivots * dim);
  const size_t o_pt = o;
  o = noalloc_align(o + sizeof(float) * gann::kPivots * dim);
  const size_t o_piv = o;
  if (piv_width) o = noalloc_align(o + sizeof(float4) * gann::kPivots * m);
  if (o > kNoallocBytes)
    return set_error(GANN_EUNSUPPORTED, "gann_search_noalloc: this index needs " + std::to_string(o) +
                                            " bytes of scratch; the static scratch holds " +
                                            std::to_string(kNoallocBytes));

  if (d->device < 0 || d->device >= kNoallocMaxDevices)
    return set_error(GANN_EUNSUPPORTED, "gann_search_noalloc: device ordinal outside 0..63");
  // the caller's current device is restored on every return path
  int prev_dev = 0;
  GANN_CUDA(cudaGetDevice(&prev_dev));
  GANN_CUDA(cudaSetDevice(d->device));
  auto on_device = [&]() -> int {
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[d->device]) {
      void* p = nullptr;
      GANN_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      g_noalloc_ptr[d->device] = static_cast<unsigned char*>(p);
    }
    base = g_noalloc_ptr[d->device];
  }
  int sm_count = 0;
  GANN_CUDA(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, d->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // stage the small tables; the counters must start at zero
  GANN_CUDA(cudaMemsetAsync(base, 0, 256, st));
  GANN_CUDA(cudaMemcpyAsync(base + o_cen, d->centroid, sizeof(float) * dim, cudaMemcpyHostToDevice, st));
  GANN_CUDA(cudaMemcpyAsync(base + o_off, off, sizeof(int32_t) * (m + 1), cudaMemcpyHostToDevice, st));
  GANN_CUDA(cudaMemcpyAsync(base + o_raw, d->pivots, sizeof(float) * gann::kPivots * dim, cudaMemcpyHostToDevice, st));
  noalloc_stage_tables<<<64, 256, 0, st>>>(reinterpret_cast<const float*>(base + o_raw),
                                           reinterpret_cast<const int32_t*>(base + o_off), dim, m, piv_width > 0,
                                           reinterpret_cast<float*>(base + o_pt),
                                           reinterpret_cast<float4*>(base + o_piv));
  GANN_CUDA(cudaGetLastError());

  DeviceIndex ix;
  ix.vecs = static_cast<const uint8_t*>(d->vectors);
  ix.adj = d->adjacency;
  ix.codes = d->codes;
  ix.pivots_t = reinterpret_cast<const float*>(base + o_pt);
  ix.centroid = reinterpret_cast<const float*>(base + o_cen);
  ix.chunk_off = reinterpret_cast<const int32_t*>(base + o_off);
  ix.n = d->num_points;
  ix.dim = dim;
  ix.degree = d->max_degree;
  ix.chunks = m;
  ix.vec_stride = d->vec_stride;
  ix.adj_stride = d->adj_stride;
  ix.code_stride = d->code_stride;
  ix.medoid = d->medoid;
  ix.metric = d->metric;
  ix.has_nav = 0;
  ix.piv4 = piv_width ? reinterpret_cast<const float4*>(base + o_piv) : nullptr;
  ix.piv_width = piv_width;
  int optin = 0;
  GANN_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d->device));
  if (gann::search_smem_bytes(ix, topk, ef_search) > static_cast<size_t>(optin))
    return set_error(GANN_EUNSUPPORTED, "gann_search_noalloc: per-query working set exceeds shared memory");
  if (nq == 0) return GANN_OK;

  gann::SearchArgs a;
  a.q = d_queries;
  a.nq = nq;
  a.topk = topk;
  a.ef = ef_search;
  a.max_hops = std::max(1 << 14, 64 * ef_search);
  a.nav_max_hops = 1 << 20;
  a.nns = d_nns;
  a.dist = d_distances;
  a.found = d_found_cnt;
  a.qcounter = reinterpret_cast<int32_t*>(base);
  a.err = reinterpret_cast<int32_t*>(base) + 1;
  GANN_CUDA(gann::launch_search(ix, a, d->dtype, sm_count, st));
  return GANN_OK;
  };
  const int rc = on_device();
  cudaSetDevice(prev_dev);
  return rc;
}
