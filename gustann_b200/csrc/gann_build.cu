// RobustPrune of many points at once, for the GPU index builder (Vamana,
// Subramanya et al., NeurIPS 2019; DiskANN's builder is absent from the
// reference, an empty submodule, so this follows the published procedure).
//
// One CTA prunes one point p: its candidates (ids sorted nearest-first, with
// their squared distances to p) are staged in shared memory with their
// vectors; the nearest live candidate c is kept, and every later live
// candidate c' with alpha * d(c, c') <= d(p, c') is dropped, until R are kept
// or none is left. uint8 distances are exact integers (dp4a); float32 ones are
// fma sums of squared differences. A second kernel sorts candidate rows by
// (distance, id) and removes repeated ids, which the builder does before
// every prune.
#include <algorithm>
#include <cstdint>

#include "gann_internal.hpp"

namespace gann {
namespace {

constexpr int kPruneThreads = 128;
constexpr int kPruneMaxK = 256;
constexpr int kPrunePad = 16;   // bytes after each staged row (bank spread)

__device__ __forceinline__ uint4 pr_load16(const uint8_t* row, int b, int rowbytes) {
  if (b + 16 <= rowbytes) return __ldg(reinterpret_cast<const uint4*>(row + b));
  uint32_t w[4] = {0, 0, 0, 0};
  for (int i = 0; i < 16 && b + i < rowbytes; ++i) w[i >> 2] |= static_cast<uint32_t>(row[b + i]) << (8 * (i & 3));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Squared L2 between two rows of `words` 16-byte words (zero padded).
template <typename T>
__device__ __forceinline__ float pr_dist(const uint8_t* a, const uint8_t* b, int words, float na, float nb) {
  if constexpr (sizeof(T) == 1) {
    uint32_t dot = 0;
    for (int w = 0; w < words; ++w) {
      const uint4 x = *reinterpret_cast<const uint4*>(a + 16 * w);
      const uint4 y = *reinterpret_cast<const uint4*>(b + 16 * w);
      dot = __dp4a(x.x, y.x, dot);
      dot = __dp4a(x.y, y.y, dot);
      dot = __dp4a(x.z, y.z, dot);
      dot = __dp4a(x.w, y.w, dot);
    }
    return static_cast<float>(static_cast<int32_t>(na) + static_cast<int32_t>(nb) - 2 * static_cast<int32_t>(dot));
  } else {
    float acc = 0.f;
    for (int w = 0; w < words; ++w) {
      const float4 x = *reinterpret_cast<const float4*>(a + 16 * w);
      const float4 y = *reinterpret_cast<const float4*>(b + 16 * w);
      float d = x.x - y.x;
      acc = __fmaf_rn(d, d, acc);
      d = x.y - y.y;
      acc = __fmaf_rn(d, d, acc);
      d = x.z - y.z;
      acc = __fmaf_rn(d, d, acc);
      d = x.w - y.w;
      acc = __fmaf_rn(d, d, acc);
    }
    return acc;
  }
}

// STAGED: candidate rows copied to shared memory (rowbytes small enough);
// otherwise they are read from global memory (L2) at every use.
template <typename T, bool STAGED>
__global__ void __launch_bounds__(kPruneThreads) prune_kernel(
    const uint8_t* __restrict__ vecs, int64_t n, int64_t stride, int dim, const int32_t* __restrict__ points,
    int64_t b, const int32_t* __restrict__ cand, const float* __restrict__ cdist, int k, int r, float alpha,
    int32_t* __restrict__ out, float* __restrict__ outd) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int rowbytes = dim * static_cast<int>(sizeof(T));
  const int words = (rowbytes + 15) / 16;
  const int srow = 16 * words + kPrunePad;
  int32_t* cid = reinterpret_cast<int32_t*>(smem);
  float* cd = reinterpret_cast<float*>(cid + kPruneMaxK);
  float* nrm = cd + kPruneMaxK;
  uint8_t* alive = reinterpret_cast<uint8_t*>(nrm + kPruneMaxK);
  int* next = reinterpret_cast<int*>(alive + kPruneMaxK);
  uint8_t* rows = reinterpret_cast<uint8_t*>(next + 4);
  const int tid = threadIdx.x;
  for (int64_t pi = blockIdx.x; pi < b; pi += gridDim.x) {
    const int32_t p = points[pi];
    for (int j = tid; j < k; j += kPruneThreads) {
      const int32_t c = cand[pi * k + j];
      const bool ok = c >= 0 && c < n && c != p;
      cid[j] = c;
      cd[j] = cdist[pi * k + j];
      alive[j] = ok;
    }
    __syncthreads();
    if (STAGED) {
      for (int i = tid; i < k * words; i += kPruneThreads) {
        const int j = i / words, w = i % words;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (alive[j]) v = pr_load16(vecs + static_cast<int64_t>(cid[j]) * stride, 16 * w, rowbytes);
        *reinterpret_cast<uint4*>(rows + j * srow + 16 * w) = v;
      }
      __syncthreads();
    }
    // uint8: integer norms for the exact ||a||^2 + ||b||^2 - 2 a.b
    if constexpr (sizeof(T) == 1) {
      for (int j = tid; j < k; j += kPruneThreads) {
        int32_t s = 0;
        if (alive[j]) {
          const uint8_t* x = STAGED ? rows + j * srow : vecs + static_cast<int64_t>(cid[j]) * stride;
          for (int d = 0; d < dim; ++d) s += static_cast<int32_t>(x[d]) * x[d];
        }
        nrm[j] = static_cast<float>(s);
      }
    }
    __syncthreads();
    int kept = 0, from = 0;
    while (kept < r) {
      // the nearest live candidate at or after `from` (first warp scans)
      if (tid < kWarp) {
        int found = k;
        for (int base = from; base < k; base += kWarp) {
          const int j = base + tid;
          const unsigned m = __ballot_sync(0xffffffffu, j < k && alive[j]);
          if (m) {
            found = base + __ffs(m) - 1;
            break;
          }
        }
        if (tid == 0) next[0] = found;
      }
      __syncthreads();
      const int c = next[0];
      if (c >= k) break;
      if (tid == 0) {
        out[pi * r + kept] = cid[c];
        outd[pi * r + kept] = cd[c];
        alive[c] = 0;
      }
      ++kept;
      from = c + 1;
      const uint8_t* xc = STAGED ? rows + c * srow : nullptr;
      for (int j = from + tid; j < k; j += kPruneThreads) {
        if (!alive[j]) continue;
        float d;
        if (STAGED) {
          d = pr_dist<T>(xc, rows + j * srow, words, nrm[c], nrm[j]);
        } else {
          // unstaged rows: fma over the elements straight from global memory
          const T* a = reinterpret_cast<const T*>(vecs + static_cast<int64_t>(cid[c]) * stride);
          const T* x = reinterpret_cast<const T*>(vecs + static_cast<int64_t>(cid[j]) * stride);
          float acc = 0.f;
          for (int e = 0; e < dim; ++e) {
            const float t = static_cast<float>(__ldg(a + e)) - static_cast<float>(__ldg(x + e));
            acc = __fmaf_rn(t, t, acc);
          }
          d = acc;
        }
        if (alpha * d <= cd[j]) alive[j] = 0;
      }
      __syncthreads();
    }
    for (int t = kept + tid; t < r; t += kPruneThreads) {
      out[pi * r + t] = -1;
      outd[pi * r + t] = INFINITY;
    }
    __syncthreads();
  }
}

// Warp bitonic sort of buf[0, p) (p a power of two, ascending).
__device__ void su_sort(uint64_t* buf, int p, int lane) {
  for (int size = 2; size <= p; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = lane; t < (p >> 1); t += kWarp) {
        const int i = 2 * t - (t & (stride - 1));
        const int j = i + stride;
        const uint64_t a = buf[i], b = buf[j];
        if ((a > b) == ((i & size) == 0)) {
          buf[i] = b;
          buf[j] = a;
        }
      }
      __syncwarp();
    }
  }
}

__device__ __forceinline__ uint32_t su_ord(float f) {
  const uint32_t b = __float_as_uint(__fadd_rn(f, 0.0f));
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float su_unord(uint32_t b) {
  return __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
}

// One warp per row: drop empty slots (id < 0) and repeated ids (the copy with
// the smallest distance stays), then sort by (distance, id); the row is
// padded with (-1, +inf).
__global__ void __launch_bounds__(128) sort_unique_kernel(const int32_t* __restrict__ ids,
                                                          const float* __restrict__ dists, int64_t rows, int k,
                                                          int p, int32_t* __restrict__ out_ids,
                                                          float* __restrict__ out_d) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp, wpb = blockDim.x / kWarp;
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem) + static_cast<size_t>(warp) * p;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * wpb + warp; r < rows; r += static_cast<int64_t>(gridDim.x) * wpb) {
    // by (id, distance): the first of each id run is its nearest copy
    for (int j = lane; j < p; j += kWarp) {
      uint64_t key = ~0ull;
      if (j < k) {
        const int32_t id = ids[r * k + j];
        if (id >= 0) key = (static_cast<uint64_t>(static_cast<uint32_t>(id)) << 32) | su_ord(dists[r * k + j]);
      }
      buf[j] = key;
    }
    __syncwarp();
    su_sort(buf, p, lane);
    // keep the first of each id, re-keyed by (distance, id): every decision
    // is read before any slot is rewritten (p <= 256: at most 8 per lane)
    uint64_t nk[kPruneMaxK / kWarp];
#pragma unroll
    for (int t = 0; t < kPruneMaxK / kWarp; ++t) {
      const int j = t * kWarp + lane;
      nk[t] = ~0ull;
      if (j < p) {
        const uint64_t a = buf[j];
        if (a != ~0ull && (j == 0 || (buf[j - 1] >> 32) != (a >> 32))) nk[t] = (a << 32) | (a >> 32);
      }
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < kPruneMaxK / kWarp; ++t) {
      const int j = t * kWarp + lane;
      if (j < p) buf[j] = nk[t];
    }
    __syncwarp();
    su_sort(buf, p, lane);
    for (int j = lane; j < k; j += kWarp) {
      const uint64_t a = buf[j];
      const bool ok = a != ~0ull;
      out_ids[r * k + j] = ok ? static_cast<int32_t>(static_cast<uint32_t>(a)) : -1;
      out_d[r * k + j] = ok ? su_unord(static_cast<uint32_t>(a >> 32)) : INFINITY;
    }
    __syncwarp();
  }
}

}  // namespace

int prune_max_candidates() { return kPruneMaxK; }

cudaError_t launch_sort_unique_rows(const int32_t* ids, const float* dists, int64_t rows, int k, int32_t* out_ids,
                                    float* out_d, int sm_count, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  int p = 1;
  while (p < k) p <<= 1;
  const size_t smem = sizeof(uint64_t) * p * 4;
  cudaError_t e = cudaFuncSetAttribute(sort_unique_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t grid = std::min<int64_t>((rows + 3) / 4, static_cast<int64_t>(sm_count) * 64);
  sort_unique_kernel<<<static_cast<unsigned>(grid), 128, smem, st>>>(ids, dists, rows, k, p, out_ids, out_d);
  return cudaGetLastError();
}

cudaError_t launch_robust_prune(const void* vecs, int64_t n, int64_t stride, int dim, int dtype,
                                const int32_t* points, int64_t b, const int32_t* cand, const float* cdist, int k,
                                int r, float alpha, int32_t* out, float* outd, int sm_count, cudaStream_t st) {
  if (b <= 0) return cudaSuccess;
  const int elem = dtype == GANN_UINT8 ? 1 : 4;
  const int words = (dim * elem + 15) / 16;
  const size_t head = kPruneMaxK * (4 + 4 + 4 + 1) + 16;
  const size_t staged = head + static_cast<size_t>(k) * (16 * words + kPrunePad);
  const bool stage = staged <= 96 * 1024;
  const size_t smem = stage ? staged : head;
  const void* v = vecs;
  auto run = [&](auto fn) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kPruneThreads, smem);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::min<int64_t>(b, static_cast<int64_t>(std::max(per_sm, 1)) * sm_count * 4);
    fn<<<static_cast<unsigned>(grid), kPruneThreads, smem, st>>>(static_cast<const uint8_t*>(v), n, stride, dim,
                                                                  points, b, cand, cdist, k, r, alpha, out, outd);
    return cudaGetLastError();
  };
  if (dtype == GANN_UINT8) return stage ? run(prune_kernel<uint8_t, true>) : run(prune_kernel<uint8_t, false>);
  return stage ? run(prune_kernel<float, true>) : run(prune_kernel<float, false>);
}

}  // namespace gann
