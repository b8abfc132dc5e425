/*
 * gann.h -- C ABI of the B200 in-HBM search path (libgann.so).
 *
 * The path: batched best-first beam search over a DiskANN/Vamana graph,
 * entered through the pivot ("nav") graph, guided by PQ asymmetric distances
 * and finished with an exact re-rank of every expanded node. Results match the
 * reference implementation (GustANN, src/impl/pure_mem.cuh:243-432) on the
 * same index files.
 *
 * Plain C types only: pointers, sizes and status codes. No torch types. A
 * handle is not re-entrant: one thread drives a handle at a time.
 *
 * Status codes replace the reference's exit(-1)/abort()/throw error paths
 * (src/layout.cpp:13-16, src/nav_graph.cu:46-49, src/ssd_search.cu:66,
 * src/common_cuda.cuh:10-17). gann_last_error() returns the message of the
 * last failing call on the calling thread.
 */
#ifndef GANN_H_
#define GANN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GANN_ABI_VERSION 1

typedef enum {
  GANN_OK = 0,
  GANN_EINVAL = 1,       /* bad argument or malformed index file        */
  GANN_EIO = 2,          /* file missing, short or unreadable           */
  GANN_ENOMEM = 3,       /* host or device allocation failed            */
  GANN_ECUDA = 4,        /* CUDA runtime error                          */
  GANN_ETIMEDOUT = 5,    /* a bounded wait gave up                      */
  GANN_EUNSUPPORTED = 6, /* mode or shape not supported by this build   */
  GANN_ESTATE = 7        /* handle used in the wrong state              */
} gann_status;

/* Element type of the stored vectors: gustann::DataType (src/common.hpp:22-25). */
typedef enum { GANN_UINT8 = 0, GANN_FLOAT = 1 } gann_dtype;

/* Distance: squared L2 (the reference's only metric, src/common.hpp:28-30) or
 * inner product, searched as the distance -<q, x> so that smaller is nearer. */
typedef enum { GANN_METRIC_L2 = 0, GANN_METRIC_IP = 1 } gann_metric;

/*
 * Index location and placement. Replaces gustann::GustANNConfig
 * (src/ssd_search.hpp:18-23) plus the use_gpu_mem flag of
 * GustANN::init_pure_mem (src/ssd_search.hpp:76).
 *   index_file        DiskANN disk index ("<prefix>_disk.index")
 *   pq_file_prefix    reads <prefix>_pivots.bin and <prefix>_compressed.bin
 *   nav_graph_prefix  directory with nav_index, nav_index.data, map.txt;
 *                     NULL or "" = enter every query at the index medoid
 *   use_gpu_mem       1: records in HBM ("-G"); 0: records in pinned host
 *                     memory, read by the GPU over the host link; 2: records
 *                     stay on storage, only the host-driven hop search
 *                     (gann_hop_*) runs -- GustANN::init_hybrid
 *   device            CUDA device ordinal
 *   layout            0 auto, 1 PQ codes only in their own array, 2 also a
 *                     copy of every node's neighbours' codes next to its
 *                     adjacency (N x R x M bytes of HBM; a hop then reads one
 *                     contiguous record). Auto builds the copy when it takes at
 *                     most a quarter of the device's memory. No counterpart in
 *                     the reference, which keeps one code array.
 *   part_count        0 or 1: every node record on this device. k > 1 (<= 8):
 *                     records split by id into k ranges of 2^s ids (the
 *                     smallest s with k * 2^s >= N), one range per device;
 *                     PQ codes, pivots and the nav graph stay whole on every
 *                     device. A hop reads its node's record from the owner's
 *                     HBM through a peer pointer (NVLink). The reference's
 *                     scale-out plan for a 1B index (records partitioned by
 *                     id range, queries sharded); the reference build itself
 *                     has no multi-GPU search.
 *   part_index        the range this handle loads (0..part_count-1); the other
 *                     ranges are attached with gann_part_attach before the
 *                     first search. -1 loads every range into its own
 *                     allocation on this device (single-device use of the
 *                     split addressing, e.g. for tests).
 *   metric            GANN_METRIC_L2 (0, the reference's) or GANN_METRIC_IP:
 *                     ADC entries, pivot-graph and exact distances all become
 *                     -<q, x> (table entry -(sum of q_i * p_ji) per chunk);
 *                     the index files are the same. No counterpart in the
 *                     reference, which is L2-only (src/common.hpp:28-30).
 */
typedef struct {
  const char* index_file;
  const char* pq_file_prefix;
  const char* nav_graph_prefix;
  int32_t dtype;
  int32_t use_gpu_mem;
  int32_t device;
  int32_t layout;
  int32_t part_count;
  int32_t part_index;
  int32_t metric;
  int32_t reserved[1];
} gann_config;

/* Replaces gustann::GustANNStats (src/ssd_search.hpp:25-27) and adds the
 * counters the HBM roofline needs. */
typedef struct {
  double run_time;        /* s: entry selection + traversal + re-rank (device) */
  double total_time;      /* s: the whole call, host copies included          */
  int64_t hops;           /* expanded nodes, summed over queries               */
  int64_t adc_evals;      /* PQ distances evaluated, summed over queries       */
  int64_t capped_queries; /* queries stopped by the hop cap (should be 0)      */
  int64_t bytes_touched;  /* algorithmic HBM bytes of this batch               */
} gann_stats;

typedef struct {
  int64_t num_points;
  int32_t dim;
  int32_t max_degree;     /* neighbour slots per record (max_m0)    */
  int32_t pq_chunks;      /* M                                      */
  int32_t dtype;
  int64_t medoid;
  int32_t node_len;       /* bytes of one on-disk record            */
  int32_t nodes_per_page;
  int32_t nav_points;     /* 0 when no nav graph                    */
  int32_t nav_start;
  int64_t device_bytes;   /* HBM held by the index                  */
} gann_info;

typedef struct gann_handle gann_handle;

/* Parse and load an index onto cfg->device. Replaces GustANN::GustANN +
 * GustANN::init_pure_mem (src/ssd_search.cu:108-112, 55-79) and the loaders
 * it calls: Layout::parse_diskann_metadata (src/layout.cpp:11-69),
 * PQSearch::read_data/init_device (src/pq_search.cu:56-185),
 * NavGraph::init (src/nav_graph.cu:41-100) and
 * PureMemExecutor::read_to_mem (src/pure_mem.cu:45-69). */
int gann_open(const gann_config* cfg, gann_handle** out);

/* Search nq queries (host buffers, row-major float32 [nq x dim]; uint8 data
 * takes its queries widened to float). Writes nns [nq x topk] (int32 ids),
 * distances [nq x topk] (squared L2, ascending) and found_cnt [nq]; slots past
 * found_cnt[i] are 0. Requires 1 <= topk <= ef_search. Synchronous.
 * Replaces GustANN::search -> PureMemExecutor::search
 * (src/ssd_search.cu:114-140, src/pure_mem.cu:71-199). stats may be NULL. */
int gann_search(gann_handle* h, const float* queries, int64_t nq, int32_t topk,
                int32_t ef_search, int32_t* nns, float* distances,
                int32_t* found_cnt, gann_stats* stats);

/* Same search on device-resident buffers (all pointers on cfg->device),
 * enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).
 * Asynchronous: no host synchronisation and no host copies. hops_out [nq]
 * (uint32, may be NULL) receives the number of expanded nodes per query.
 * Same kernel path as gann_search (src/pure_mem.cu:101-187 is the span it
 * replaces); the caller owns the buffers. */
int gann_search_device(gann_handle* h, const float* d_queries, int64_t nq,
                       int32_t topk, int32_t ef_search, int32_t* d_nns,
                       float* d_distances, int32_t* d_found_cnt,
                       uint32_t* d_hops_out, void* stream);

/*
 * A device-resident index the caller owns (no files): the arrays stay where
 * the caller put them and must outlive the handle; the caller may rewrite
 * `adjacency` between searches (an index builder refining its graph does).
 * Layouts (all rows 16-byte aligned):
 *   vectors    [n x vec_stride bytes], `dim` elements of `dtype` per row
 *   adjacency  [n x adj_stride] uint32 neighbour ids, unused slots 0xffffffff
 *   codes      [n x code_stride] uint8 PQ codes, code_stride % 16 == 0
 * pivots [256 x dim], centroid [dim] and chunk_offsets [pq_chunks + 1] are host
 * arrays in the PQ-file layout; they are copied. Searches enter at `medoid`.
 * No counterpart in the reference, whose indexes are always loaded from files
 * (src/ssd_search.cu:55-79); it serves graph construction on the GPU.
 */
typedef struct {
  const void* vectors;
  int64_t vec_stride;
  const uint32_t* adjacency;
  int32_t adj_stride;
  int32_t max_degree;
  const uint8_t* codes;
  int32_t code_stride;
  int32_t pq_chunks;
  const float* pivots;
  const float* centroid;
  const uint32_t* chunk_offsets;
  int64_t num_points;
  int32_t dim;
  int32_t dtype;
  int64_t medoid;
  int32_t device;
  int32_t metric;          /* GANN_METRIC_L2 or GANN_METRIC_IP, as gann_config */
  int32_t reserved[2];
} gann_device_index;

int gann_open_device(const gann_device_index* desc, gann_handle** out);

/*
 * Allocation-free search. For callers that cannot call cudaMalloc on the
 * search path -- a serving process whose HBM is handed out by another runtime's
 * arena, or a caller that must not trigger the allocator's device-wide
 * synchronisation while other work is in flight. It searches the caller-owned
 * device index described by `desc` (the gann_open_device layout) for queries
 * and outputs the caller also owns, and allocates nothing: the library-side
 * device state of the call -- the work and error counters, and the centroid,
 * chunk offsets and PQ pivot tables staged from desc's host arrays -- lives in
 * one static device array of GANN_NOALLOC_SCRATCH_BYTES (1 MiB) that every GPU
 * loading the library holds until exit. The table space needed is about
 * 2048*dim + 4096*pq_chunks bytes; an index needing more than the array is
 * rejected with GANN_EUNSUPPORTED. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) and keeps it for the life of
 * the process; that first call on a device should come before any stream
 * capture. The address belongs to the device's primary context: call from
 * that context, and a cudaDeviceReset ends the array's use by this entry
 * point for the process.
 * All calls share the one array and each call re-stages it, so calls whose
 * work overlaps on the GPU race: serialise them (one stream, or wait for the
 * previous call). Asynchronous on `stream`: desc's host arrays (pivots,
 * centroid, chunk offsets) are read by copies enqueued on the stream; ordinary
 * pageable arrays may be reused when the call returns, page-locked ones must
 * stay unchanged until the stream has passed the call. Results are the same as
 * gann_search_device over the same arrays. Queries stopped by the hop cap are
 * not reported by this entry point (it has no statistics output). The
 * caller's current device is left as it was.
 * No counterpart in the reference, which allocates per search call
 * (src/pure_mem.cu:78-89).
 */
#define GANN_NOALLOC_SCRATCH_BYTES (1u << 20)
int gann_search_noalloc(const gann_device_index* desc, const float* d_queries, int64_t nq,
                        int32_t topk, int32_t ef_search, int32_t* d_nns, float* d_distances,
                        int32_t* d_found_cnt, void* stream);

/*
 * Partitioned records across processes (one process per GPU). gann_part_export
 * writes, into `blob` (GANN_PART_BLOB_BYTES), CUDA IPC handles of the handle's
 * own record range; another process passes that blob to gann_part_attach with
 * the range's index, which maps the range into its address space (peer access
 * over NVLink is enabled on first use). Search returns GANN_ESTATE until every
 * range is present. Attached ranges are unmapped by gann_close. Blobs are
 * opaque and valid while the exporting handle is open.
 */
#define GANN_PART_BLOB_BYTES 512
int gann_part_export(gann_handle* h, void* blob, int64_t blob_bytes);
int gann_part_attach(gann_handle* h, int32_t part, const void* blob, int64_t blob_bytes);

/*
 * Host-driven search, one hop per call: the reference's SSD-hybrid mode
 * (GustANN::init_hybrid + HybridExecutor, src/hybrid.cu; per-hop kernels
 * src/impl/hyd_search_v2.cuh:8-472 driven by src/hyd_task_runner.cu:12-329),
 * for indexes whose node records stay on storage. PQ codes, pivots and the
 * pivot graph are in HBM (a handle opened as usual); the caller reads, between
 * hops, the 4 KB page that holds each query's requested node -- page
 * 1 + id / nodes_per_page of the disk index (gann_read_pages does this with
 * pread) -- and hands the pages to gann_hop_step. As in the reference's hybrid
 * mode, the pivot-graph entry and the re-rank use q'' = (q - c) + c.
 *   gann_hop_begin     stage nq queries (host, float32 [nq x dim]); entries found
 *   gann_hop_requests  node id each query needs next, -1 when it is done
 *                      (host int32 [nq]); *active = number of ids >= 0
 *   gann_hop_step      advance every active query by one hop; pages = host
 *                      [nq x 4096] with row i = the page of node_ids[i] (rows of
 *                      finished queries are ignored)
 *   gann_hop_finish    results, as gann_search writes them
 *   gann_hop_free      release the batch (the handle stays open)
 * Needs dim * element size and the record length to be multiples of 4 bytes.
 * The handle must outlive its batches. Several batches of one handle may be
 * open at once (each holds its own device state); calls on a handle and its
 * batches must not run concurrently from several threads (gann_read_pages,
 * which takes no handle, may).
 */
typedef struct gann_hop_batch gann_hop_batch;
int gann_hop_begin(gann_handle* h, const float* queries, int64_t nq, int32_t topk, int32_t ef_search,
                   gann_hop_batch** out);
int gann_hop_requests(gann_hop_batch* b, int32_t* node_ids, int64_t* active);
int gann_hop_step(gann_hop_batch* b, const void* pages);
int gann_hop_finish(gann_hop_batch* b, int32_t* nns, float* distances, int32_t* found_cnt);
int gann_hop_free(gann_hop_batch* b);

/* Storage loader for the host-driven search: reads, for each of n node ids,
 * the 4 KB page holding its record from a disk index (page 1 + id /
 * nodes_per_page) into pages[i * 4096], with `threads` reader threads (<= 0:
 * hardware concurrency). Ids < 0 leave their row untouched. Host only. Takes
 * the place of the reference's IO backends for a file on a local disk
 * (src/io/interface.hpp:10-40, src/io/mem_io.cpp:11-51). */
int gann_read_pages(const char* index_file, const int32_t* node_ids, int64_t n, int32_t nodes_per_page,
                    void* pages, int32_t threads);

/* Release device and host memory of the handle (GustANN::~GustANN,
 * src/ssd_search.cu:112-137). NULL is accepted. */
int gann_close(gann_handle* h);

/* Tuning options (no counterpart in the reference).
 *   GANN_OPT_ADC_MODE: 0 auto, 1 per-query ADC table in shared memory, 2 the
 *     PQ pivot table resident once per SM with table entries recomputed per
 *     lookup (bit-identical sums; needs <= 4 dims per chunk and D <= 128),
 *     3 filtered: a per-query table of 8-bit lower bounds of the entries
 *     rejects the candidates a full pool would cut anyway, and only the rest
 *     get their exact ADC, recomputed from the pivot rows (bit-identical
 *     results; L2, <= 4 dims per chunk, <= 32 chunks, D <= 128).
 *     Auto picks 2 when it fits.
 *   GANN_OPT_PIVOT_WARPS: queries in flight per SM in modes 2 and 3 (8..24,
 *     0 auto).
 *   GANN_OPT_NEIGHBOUR_CODES: 1 read neighbour codes from the per-node copy
 *     when the handle has one (layout 0/2), 0 from the shared code array. */
enum { GANN_OPT_ADC_MODE = 1, GANN_OPT_PIVOT_WARPS = 2, GANN_OPT_NEIGHBOUR_CODES = 3 };
int gann_set_option(gann_handle* h, int32_t option, int64_t value);

/* Message of the last failed call on this thread ("" if none). */
const char* gann_last_error(void);

int gann_index_info(const gann_handle* h, gann_info* out);

/* Stage probes (test hooks on the same device functions as the search):
 *   gann_probe_lut: per-query ADC tables [nq x M x 256] float32, the
 *     PQSearchData::init_query table (src/impl/pq.cuh:8-59);
 *   gann_probe_entry: per-query nav result as sample index and as global id
 *     (get_entry_kernel_inner + NavGraph::translate, src/impl/nav.cuh:13-135,
 *     src/nav_graph.cu:104-109). Host buffers, synchronous. */
int gann_probe_lut(gann_handle* h, const float* queries, int64_t nq, float* luts);
int gann_probe_entry(gann_handle* h, const float* queries, int64_t nq,
                     int32_t* sample_idx, int32_t* entry_ids);

/* Pivot-graph sample: the sorted first `s` ids of a std::shuffle of [0, n)
 * driven by std::mt19937(seed) -- the sampling step of bin/gen_small_file.cpp:18-40
 * (seed 114514 there). Host only. */
int gann_pivot_sample(int64_t n, int64_t s, uint32_t seed, int32_t* out);

/* Exact k nearest neighbours by brute force on the GPU: the ground truth that
 * recall@k is computed against (the reference reads it from an ivecs file,
 * bin/search_disk.cpp:206-213, and computes recall with calc_recall,
 * bin/utils.hpp:104-116; the file itself comes from tools outside the
 * reference). Device buffers on `device`, enqueued on `stream`:
 *   base      [num_points rows x base_stride bytes], `dim` elements of dtype
 *   queries   [nq rows x query_stride bytes], same dtype as the base (uint8
 *             queries as uint8); strides and both pointers 16-byte aligned
 *   ids       [nq x k] int32, distances [nq x k] float32, ascending by
 *             (distance, id); L2 distances are squared (exact integers for
 *             uint8 data), IP distances are -<q, x>.
 * 1 <= k <= 128. Allocates temporary device memory on the stream
 * (cudaMallocAsync). */
int gann_exact_knn(const void* d_base, int64_t num_points, int64_t base_stride, int32_t dim, int32_t dtype,
                   const void* d_queries, int64_t query_stride, int64_t nq, int32_t k, int32_t metric,
                   int32_t* d_ids, float* d_distances, int32_t device, void* stream);

/* RobustPrune (Subramanya et al., NeurIPS 2019) of `count` points at once, for
 * building the graph the search runs on (the reference takes its indexes from
 * DiskANN's builder, an empty submodule in its tree). Point i = points[i] has
 * `k` candidates cand[i * k ..] sorted nearest-first (-1 = empty), with their
 * squared L2 distances cand_dist[i * k ..] to the point; the nearest live
 * candidate c is kept and every later live candidate c' with
 * alpha * |c - c'|^2 <= cand_dist(c') is dropped, until r are kept. Writes
 * out [count x r] int32 (nearest-first, -1 padded) and out_dist [count x r]
 * (+inf padded). Device buffers on `device`, enqueued on `stream`; vectors
 * [num_points rows x stride bytes] of dtype, 16-byte aligned. k <= 256. */
int gann_robust_prune(const void* d_vectors, int64_t num_points, int64_t stride, int32_t dim, int32_t dtype,
                      const int32_t* d_points, int64_t count, const int32_t* d_cand, const float* d_cand_dist,
                      int32_t k, int32_t r, float alpha, int32_t* d_out, float* d_out_dist, int32_t device,
                      void* stream);

/* Candidate rows for gann_robust_prune: each of `rows` rows of `k` (id,
 * distance) pairs is sorted by (distance, id) with empty slots (id < 0) and
 * repeated ids removed (the nearest copy stays), padded with (-1, +inf).
 * Device buffers, k <= 256; out may not alias in. No counterpart in the
 * reference (index construction is DiskANN's there). */
int gann_sort_unique_rows(const int32_t* d_ids, const float* d_dists, int64_t rows, int32_t k, int32_t* d_out_ids,
                          float* d_out_dists, int32_t device, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GANN_H_ */
