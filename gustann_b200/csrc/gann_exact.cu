// Exact k-nearest-neighbour search by brute force: the ground truth that
// recall@k is measured against (the reference reads it from an ivecs file made
// by external tools, bin/search_disk.cpp:206-213, bin/utils.hpp:104-116).
//
// One CTA holds 32 queries in shared memory and streams a slice of the base
// points through a double-buffered shared-memory tile of 128 points x 128
// bytes; every warp owns 4 queries and computes their 4 x 128 dot products of
// the tile (lane = 4 points), uint8 rows with dp4a (exact integer sums), float
// rows with fma. Distances are
//   L2  ||q||^2 + ||x||^2 - 2 q.x   (exact for uint8 data: integers < 2^24)
//   IP  -q.x
// and a candidate enters its query's buffer when its 64-bit key
// (ord(dist) << 32 | id) is below the query's current k-th best key; a full
// buffer is sorted in place (bitonic, by the owning warp) and cut to k. The
// grid splits the points into slices when the queries alone do not fill the
// GPU; a second kernel merges the slices' top-k lists per query.
#include <algorithm>
#include <cstdint>

#include "gann_internal.hpp"

namespace gann {
namespace {

constexpr int kExQ = 32;        // queries per CTA
constexpr int kExP = 128;       // points per tile
constexpr int kExRow = 128;     // bytes of a row per tile chunk
constexpr int kExPad = 16;      // row padding in shared memory (bank spread)
constexpr int kExThreads = 256; // 8 warps x 4 queries
constexpr unsigned kExFull = 0xffffffffu;

__device__ __forceinline__ uint32_t ex_ord(float f) {
  uint32_t b = __float_as_uint(__fadd_rn(f, 0.0f));
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ex_unord(uint32_t b) {
  return __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
}

// 16 bytes of a row, zero past `rowbytes` (rows need not be a multiple of 16 B).
__device__ __forceinline__ uint4 ex_load16(const uint8_t* row, int64_t b, int64_t rowbytes) {
  if (b + 16 <= rowbytes) return __ldg(reinterpret_cast<const uint4*>(row + b));
  uint32_t w[4] = {0, 0, 0, 0};
  for (int i = 0; i < 16 && b + i < rowbytes; ++i) w[i >> 2] |= static_cast<uint32_t>(row[b + i]) << (8 * (i & 3));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
struct ExAcc;
template <>
struct ExAcc<uint8_t> {
  using type = uint32_t;
  __device__ static void dot(uint32_t& a, const uint4& x, const uint4& y) {
    a = __dp4a(x.x, y.x, a);
    a = __dp4a(x.y, y.y, a);
    a = __dp4a(x.z, y.z, a);
    a = __dp4a(x.w, y.w, a);
  }
  __device__ static float dist(uint32_t acc, float qn, float pn, bool ip) {
    if (ip) return -static_cast<float>(acc);
    const int32_t d = static_cast<int32_t>(qn) + static_cast<int32_t>(pn) - 2 * static_cast<int32_t>(acc);
    return static_cast<float>(d);
  }
};
template <>
struct ExAcc<float> {
  using type = float;
  __device__ static void dot(float& a, const uint4& x, const uint4& y) {
    a = __fmaf_rn(__uint_as_float(x.x), __uint_as_float(y.x), a);
    a = __fmaf_rn(__uint_as_float(x.y), __uint_as_float(y.y), a);
    a = __fmaf_rn(__uint_as_float(x.z), __uint_as_float(y.z), a);
    a = __fmaf_rn(__uint_as_float(x.w), __uint_as_float(y.w), a);
  }
  __device__ static float dist(float acc, float qn, float pn, bool ip) {
    if (ip) return -acc;
    return fmaxf(qn + pn - 2.f * acc, 0.f);
  }
};

// Bitonic sort of buf[0, p) (p a power of two) by one warp.
__device__ void ex_warp_sort(uint64_t* buf, int p, int lane) {
  for (int size = 2; size <= p; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = lane; t < (p >> 1); t += kWarp) {
        const int i = 2 * t - (t & (stride - 1));
        const int j = i + stride;
        const uint64_t a = buf[i], b = buf[j];
        const bool up = (i & size) == 0;
        if ((a > b) == up) {
          buf[i] = b;
          buf[j] = a;
        }
      }
      __syncwarp();
    }
  }
}

__device__ __forceinline__ int ex_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Sort a query's candidate buffer and keep its `k` best keys; returns the new
// threshold key (the k-th best, or all-ones while fewer than k were seen).
__device__ uint64_t ex_compact(uint64_t* buf, int& cnt, int k, int lane) {
  const int p = ex_pow2(max(cnt, 2));
  for (int i = cnt + lane; i < p; i += kWarp) buf[i] = ~0ull;
  __syncwarp();
  ex_warp_sort(buf, p, lane);
  cnt = min(cnt, k);
  return cnt == k ? buf[k - 1] : ~0ull;
}

template <typename T>
__global__ void __launch_bounds__(256) point_norms(const uint8_t* __restrict__ base, int64_t n, int64_t stride,
                                                   int dim, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const T* r = reinterpret_cast<const T*>(base + i * stride);
    if constexpr (sizeof(T) == 1) {
      int32_t s = 0;
      for (int d = 0; d < dim; ++d) s += static_cast<int32_t>(r[d]) * r[d];
      out[i] = static_cast<float>(s);
    } else {
      float s = 0.f;
      for (int d = 0; d < dim; ++d) s = __fmaf_rn(r[d], r[d], s);
      out[i] = s;
    }
  }
}

// Shared-memory layout of one CTA (mirrored by ex_smem_bytes).
struct ExSmem {
  uint8_t* qs;      // [kExQ][qrow]  query rows, zero padded
  uint8_t* ps;      // [2][kExP][kExRow + kExPad]
  uint64_t* cand;   // [kExQ][cap]
  float* qn;        // [kExQ]
};

__host__ __device__ inline size_t ex_smem_bytes(int64_t qrow, int cap) {
  return static_cast<size_t>(kExQ) * qrow + 2 * kExP * (kExRow + kExPad) + static_cast<size_t>(kExQ) * cap * 8 +
         kExQ * sizeof(float);
}

template <typename T>
__global__ void __launch_bounds__(kExThreads) exact_knn_kernel(
    const uint8_t* __restrict__ base, int64_t n, int64_t bstride, int dim, const uint8_t* __restrict__ queries,
    int64_t qstride, int64_t nq, int k, int kpad, int cap, int slices, int ip, const float* __restrict__ pnorm,
    uint64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  using Acc = ExAcc<T>;
  using A = typename Acc::type;
  const int64_t rowbytes = static_cast<int64_t>(dim) * sizeof(T);
  const int nch = static_cast<int>((rowbytes + kExRow - 1) / kExRow);
  const int64_t qrow = static_cast<int64_t>(nch) * kExRow;
  ExSmem s;
  s.qs = smem;
  s.ps = s.qs + kExQ * qrow;
  s.cand = reinterpret_cast<uint64_t*>(s.ps + 2 * kExP * (kExRow + kExPad));
  s.qn = reinterpret_cast<float*>(s.cand + static_cast<size_t>(kExQ) * cap);
  const int tid = threadIdx.x, lane = tid % kWarp, warp = tid / kWarp;
  const int64_t qt = blockIdx.x / slices;
  const int slice = blockIdx.x % slices;
  const int64_t q0 = qt * kExQ;

  // query rows (zero padded to whole chunks) and their norms
  for (int64_t i = tid; i < kExQ * qrow / 16; i += kExThreads) {
    const int64_t r = i / (qrow / 16), b = (i % (qrow / 16)) * 16;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q0 + r < nq) v = ex_load16(queries + (q0 + r) * qstride, b, rowbytes);
    *reinterpret_cast<uint4*>(s.qs + r * qrow + b) = v;
  }
  __syncthreads();
  if (tid < kExQ) {
    const T* r = reinterpret_cast<const T*>(s.qs + tid * qrow);
    float acc = 0.f;
    if constexpr (sizeof(T) == 1) {
      int32_t a = 0;
      for (int d = 0; d < dim; ++d) a += static_cast<int32_t>(r[d]) * r[d];
      acc = static_cast<float>(a);
    } else {
      for (int d = 0; d < dim; ++d) acc = __fmaf_rn(r[d], r[d], acc);
    }
    s.qn[tid] = acc;
  }
  // this warp's 4 queries: candidate buffers, counts and thresholds
  int cnt[4] = {0, 0, 0, 0};
  uint64_t thr[4] = {~0ull, ~0ull, ~0ull, ~0ull};
  bool qvalid[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qvalid[i] = q0 + 4 * warp + i < nq;
  __syncthreads();

  const int64_t per = ((n + slices - 1) / slices + kExP - 1) / kExP * kExP;
  const int64_t pbeg = slice * per, pend = min(n, pbeg + per);
  const int64_t ntiles = pbeg < pend ? (pend - pbeg + kExP - 1) / kExP : 0;
  const int64_t steps = ntiles * nch;

  // tile chunk loads: 128 rows x 8 uint4, 4 per thread
  uint4 reg[4];
  auto load_chunk = [&](int64_t step) {
    const int64_t tile = step / nch;
    const int c = static_cast<int>(step % nch);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = tid + kExThreads * r;
      const int row = i >> 3, col = (i & 7) * 16;
      const int64_t p = pbeg + tile * kExP + row;
      reg[r] = p < pend ? ex_load16(base + p * bstride, static_cast<int64_t>(c) * kExRow + col, rowbytes)
                        : make_uint4(0, 0, 0, 0);
    }
  };
  if (steps > 0) load_chunk(0);
  A acc[4][4];
  for (int64_t st = 0; st < steps; ++st) {
    const int c = static_cast<int>(st % nch);
    uint8_t* buf = s.ps + (st & 1) * kExP * (kExRow + kExPad);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = tid + kExThreads * r;
      *reinterpret_cast<uint4*>(buf + (i >> 3) * (kExRow + kExPad) + (i & 7) * 16) = reg[r];
    }
    __syncthreads();
    if (st + 1 < steps) load_chunk(st + 1);
    if (c == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = A(0);
    }
#pragma unroll
    for (int kk = 0; kk < kExRow / 16; ++kk) {
      uint4 qv[4], pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qv[i] = *reinterpret_cast<const uint4*>(s.qs + (4 * warp + i) * qrow + c * kExRow + kk * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pv[j] = *reinterpret_cast<const uint4*>(buf + (lane + kWarp * j) * (kExRow + kExPad) + kk * 16);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) Acc::dot(acc[i][j], qv[i], pv[j]);
    }
    if (c == nch - 1) {
      const int64_t tbase = pbeg + (st / nch) * kExP;
      float pn[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t p = tbase + lane + kWarp * j;
        pn[j] = (!ip && p < pend) ? __ldg(pnorm + p) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int qi = 4 * warp + i;
        uint64_t* cb = s.cand + static_cast<size_t>(qi) * cap;
        const float qn = s.qn[qi];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t p = tbase + lane + kWarp * j;
          const uint64_t key = (static_cast<uint64_t>(ex_ord(Acc::dist(acc[i][j], qn, pn[j], ip))) << 32) |
                               static_cast<uint32_t>(p);
          const bool take = qvalid[i] && p < pend && key < thr[i];
          const unsigned bm = __ballot_sync(kExFull, take);
          if (take) cb[cnt[i] + __popc(bm & ((1u << lane) - 1u))] = key;
          cnt[i] += __popc(bm);
        }
        __syncwarp();
        // a buffer that another tile could overflow is cut back to k
        if (cnt[i] > cap - kExP) thr[i] = ex_compact(cb, cnt[i], k, lane);
      }
    }
  }
  // this slice's top-k of every query, padded with all-ones keys
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t q = q0 + 4 * warp + i;
    if (q >= nq) continue;
    uint64_t* cb = s.cand + static_cast<size_t>(4 * warp + i) * cap;
    ex_compact(cb, cnt[i], k, lane);
    uint64_t* o = out + (q * slices + slice) * kpad;
    for (int t = lane; t < kpad; t += kWarp) o[t] = t < cnt[i] ? cb[t] : ~0ull;
  }
}

// Merge the slices' lists of each query (one warp per query) into ids and
// distances, ascending by (distance, id); missing entries are id -1, +inf.
__global__ void __launch_bounds__(128) exact_merge_kernel(const uint64_t* __restrict__ part, int64_t nq, int slices,
                                                          int kpad, int k, int32_t* __restrict__ ids,
                                                          float* __restrict__ dists) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp, wpb = blockDim.x / kWarp;
  const int total = slices * kpad;
  const int p = ex_pow2(max(total, 2));
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem) + static_cast<size_t>(warp) * p;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * wpb + warp; q < nq; q += static_cast<int64_t>(gridDim.x) * wpb) {
    for (int i = lane; i < p; i += kWarp) buf[i] = i < total ? part[q * total + i] : ~0ull;
    __syncwarp();
    if (slices > 1) ex_warp_sort(buf, p, lane);
    for (int t = lane; t < k; t += kWarp) {
      const uint64_t key = buf[t];
      const bool ok = key != ~0ull;
      ids[q * k + t] = ok ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
      dists[q * k + t] = ok ? ex_unord(static_cast<uint32_t>(key >> 32)) : INFINITY;
    }
    __syncwarp();
  }
}

}  // namespace

int exact_knn_max_k() { return 128; }

cudaError_t launch_exact_knn(const void* base, int64_t n, int64_t bstride, int dim, int dtype, const void* queries,
                             int64_t qstride, int64_t nq, int k, int metric, int32_t* ids, float* dists,
                             int sm_count, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  const int64_t rowbytes = static_cast<int64_t>(dim) * (dtype == GANN_UINT8 ? 1 : 4);
  const int64_t qrow = (rowbytes + kExRow - 1) / kExRow * kExRow;
  const int kpad = (k + kWarp - 1) / kWarp * kWarp;
  int cap = 1;
  while (cap < kpad + kExP) cap <<= 1;
  const size_t smem = ex_smem_bytes(qrow, cap);
  auto fn = dtype == GANN_UINT8 ? exact_knn_kernel<uint8_t> : exact_knn_kernel<float>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kExThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  const int64_t qt = (nq + kExQ - 1) / kExQ;
  const int64_t slots = static_cast<int64_t>(per_sm) * sm_count;
  // slices so that the grid covers the GPU a few times over
  int slices = static_cast<int>(std::min<int64_t>(32, std::max<int64_t>(1, (4 * slots + qt - 1) / qt)));
  slices = static_cast<int>(std::min<int64_t>(slices, std::max<int64_t>(1, (n + kExP - 1) / kExP)));
  float* pn = nullptr;
  uint64_t* part = nullptr;
  if (metric == GANN_METRIC_L2) {
    e = cudaMallocAsync(reinterpret_cast<void**>(&pn), sizeof(float) * static_cast<size_t>(n), st);
    if (e != cudaSuccess) return e;
    const unsigned g = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 32));
    if (dtype == GANN_UINT8)
      point_norms<uint8_t><<<g, 256, 0, st>>>(static_cast<const uint8_t*>(base), n, bstride, dim, pn);
    else
      point_norms<float><<<g, 256, 0, st>>>(static_cast<const uint8_t*>(base), n, bstride, dim, pn);
  }
  e = cudaMallocAsync(reinterpret_cast<void**>(&part), sizeof(uint64_t) * static_cast<size_t>(nq) * slices * kpad, st);
  if (e == cudaSuccess) {
    fn<<<static_cast<unsigned>(qt * slices), kExThreads, smem, st>>>(
        static_cast<const uint8_t*>(base), n, bstride, dim, static_cast<const uint8_t*>(queries), qstride, nq, k, kpad,
        cap, slices, metric == GANN_METRIC_IP, pn, part);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    int pw = 1;
    while (pw < slices * kpad) pw <<= 1;
    const size_t msmem = sizeof(uint64_t) * pw * 4;
    e = cudaFuncSetAttribute(exact_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(msmem));
    if (e == cudaSuccess) {
      const unsigned g = static_cast<unsigned>(std::min<int64_t>((nq + 3) / 4, 148 * 64));
      exact_merge_kernel<<<g, 128, msmem, st>>>(part, nq, slices, kpad, k, ids, dists);
      e = cudaGetLastError();
    }
  }
  if (part) cudaFreeAsync(part, st);
  if (pn) cudaFreeAsync(pn, st);
  return e;
}

}  // namespace gann
