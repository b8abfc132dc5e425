// Fused search kernel for sm_100a: one warp owns one query at a time and runs
// entry selection on the pivot graph, the ADC table build, the best-first
// traversal and the exact re-rank without leaving the SM.
//
// Results equal the reference's (src/impl/pure_mem.cuh:243-432 with
// src/impl/nav.cuh:13-135 and src/impl/pq.cuh:8-59) on the same inputs. The
// floating-point operations that decide the traversal are issued in the
// reference's order:
//   * ADC table entry: per chunk, dims ascending, acc = fma(d, d, acc) from 0
//     with d = (q_i - centroid_i) - pivot_ji          (src/impl/pq.cuh:22-43)
//   * ADC distance: sequential fp32 adds over chunks 0..M-1
//                                                     (src/impl/pure_mem.cuh:303-308)
//   * exact distance: lane-strided fma partial sums, then the shfl_down tree
//     16/8/4/2/1 (src/impl/util.cuh:26-46), on q'' = (q - c) + c for the
//     traversal re-rank and on q for the pivot graph.
// With the inner-product metric (no counterpart in the reference, which is
// L2-only: src/common.hpp:28-30) every distance is -<q, x>: table entries
// -(fma chain of q_i * p_ji from 0 over the chunk's dims), exact distances the
// same lane-strided fma sums and shfl_down tree on q . x, negated; q'' = q.
// Candidate order is the total order (distance, id & 0x7fffffff)
// (src/impl/util.cuh:166-178); the pool keeps the first `ef` distinct entries
// of merge(pool, neighbours) with the pool copy first on equal keys, which is
// what the reference's merge + 2L cut + dedup produce
// (src/impl/pure_mem.cuh:350-419).
#include <algorithm>
#include <cstdint>
#include <climits>

#include "gann_internal.hpp"

namespace gann {
namespace {

constexpr unsigned kFull = 0xffffffffu;

// Distances become the high word of a 64-bit sort key. Adding +0.0f folds -0
// into +0, because the reference compares distances with < and ==.
__device__ __forceinline__ uint32_t ord_f32(float f) {
  uint32_t b = __float_as_uint(__fadd_rn(f, 0.0f));
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Pool / candidate key: [ord(dist) : 32][id : 31][unvisited : 1]. Comparing
// key >> 1 compares (dist, id); a visited pool copy sorts before an unvisited
// copy of the same node.
__device__ __forceinline__ uint64_t make_key(float d, uint32_t id) {
  return (static_cast<uint64_t>(ord_f32(d)) << 32) | (static_cast<uint64_t>(id) << 1) | 1ull;
}

template <typename T>
__device__ __forceinline__ void load32(const T* __restrict__ p, float (&v)[32]);

template <>
__device__ __forceinline__ void load32<uint8_t>(const uint8_t* __restrict__ p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  uint4 a = __ldg(q), b = __ldg(q + 1);
  uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = static_cast<float>((w[i >> 2] >> (8 * (i & 3))) & 0xffu);
}

template <>
__device__ __forceinline__ void load32<float>(const float* __restrict__ p, float (&v)[32]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 t = __ldg(q + i);
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
}

// One lane's term of an exact distance: squared difference, or the product
// for the inner product.
template <bool IP>
__device__ __forceinline__ float dist_acc(float q, float x, float acc) {
  if (IP) return __fmaf_rn(q, x, acc);
  const float d = __fsub_rn(q, x);
  return __fmaf_rn(d, d, acc);
}

// Exact distance with the reference's warp order: lane l sums dims l, l+32, ...
// with fma, then the shfl_down tree (src/impl/util.cuh:26-46); negated for the
// inner product. All lanes get lane 0's value.
template <typename T, bool IP>
__device__ __forceinline__ float warp_dist(const float* __restrict__ qv, const T* __restrict__ x,
                                           int dim, int lane) {
  float acc = 0.f;
  for (int i = lane; i < dim; i += kWarp) acc = dist_acc<IP>(qv[i], static_cast<float>(x[i]), acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, off));
  const float r = __shfl_sync(kFull, acc, 0);
  return IP ? -r : r;
}

// The same value computed by ONE lane for a whole vector: the 32 lane partials
// live in registers and the shfl_down tree is replayed (lane 0's sum at every
// level), so 28 pivot-graph neighbours are measured at once, one per lane.
template <typename T, bool IP>
__device__ __forceinline__ float lane_dist(const float* __restrict__ qv, const T* __restrict__ x,
                                           int dim) {
  float p[32];
#pragma unroll
  for (int m = 0; m < 32; ++m) p[m] = 0.f;
  for (int base = 0; base < dim; base += 32) {
    float xv[32];
    load32<T>(x + base, xv);
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      if (base + m < dim) p[m] = dist_acc<IP>(qv[base + m], xv[m], p[m]);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int m = 0; m < off; ++m) p[m] = __fadd_rn(p[m], p[m + off]);
  }
  return IP ? -p[0] : p[0];
}

// Greedy entry search on the pivot graph (src/impl/nav.cuh:13-135), lane = slot.
// Slots [0,4) hold the best entries, [4,32) the neighbours of the last expanded
// node; slots past the neighbour count keep stale entries, as in the reference.
// Returns the sample index of slot 0.
template <typename T, bool IP>
__device__ int nav_search(const DeviceIndex& ix, const float* __restrict__ qs, int lane,
                          int max_hops, bool& capped) {
  const T* nv = reinterpret_cast<const T*>(ix.nav_vecs);
  const size_t rs = static_cast<size_t>(ix.nav_stride) / sizeof(T);
  const int start = ix.nav_start;
  const float d0 = warp_dist<T, IP>(qs, nv + static_cast<size_t>(start) * rs, ix.dim, lane);
  uint32_t sid = lane == 0 ? static_cast<uint32_t>(start) : kPadId;
  float sd = lane == 0 ? d0 : INFINITY;
  int idx = 0;
  for (int hop = 0;; ++hop) {
    if (hop >= max_hops) {
      capped = true;
      break;
    }
    const uint32_t u = __shfl_sync(kFull, sid, idx);
    if (lane == idx) sid |= kVisited;
    const int v = lane < kNavNbr ? __ldg(ix.nav_adj + static_cast<size_t>(u) * ix.nav_row + lane) : -1;
    // the neighbour list ends at the first -1 or after 28 entries
    const unsigned term = __ballot_sync(kFull, lane >= kNavNbr || v == -1);
    const int cnt = __ffs(term) - 1;
    float dv = INFINITY;
    if (lane < cnt) dv = lane_dist<T, IP>(qs, nv + static_cast<size_t>(v) * rs, ix.dim);
    const int src = lane >= kNavBest ? lane - kNavBest : 0;
    const uint32_t nid = __shfl_sync(kFull, static_cast<uint32_t>(v), src);
    const float nd = __shfl_sync(kFull, dv, src);
    if (lane >= kNavBest && lane - kNavBest < cnt) {
      sid = nid;
      sd = nd;
    }
#pragma unroll
    for (int i = 0; i < kNavBest; ++i) {
      const uint32_t prev = __shfl_sync(kFull, sid, i > 0 ? i - 1 : 0);
      float dist = sd;
      int pos = lane;
      bool kill = false;
      if (lane < i) dist = INFINITY;
      else if (i != 0 && ((sid ^ prev) & 0x7fffffffu) == 0) kill = true;
      // A copy of slot i-1's node is dropped and its visited bit folded into
      // slot i-1. With several copies in one round the reference's stores race;
      // the highest lane's value is taken here.
      const unsigned km = __ballot_sync(kFull, kill);
      if (km) {
        const uint32_t hv = __shfl_sync(kFull, sid, 31 - __clz(km));
        if (lane == i - 1) sid = prev | hv;
      }
      if (kill) {
        sd = INFINITY;
        dist = INFINITY;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const int op = __shfl_down_sync(kFull, pos, off);
        const float ov = __shfl_down_sync(kFull, dist, off);
        if (ov < dist) {
          dist = ov;
          pos = op;
        }
      }
      pos = __shfl_sync(kFull, pos, 0);
      if (i != pos) {
        const float t = __shfl_sync(kFull, sd, i);
        const float y = __shfl_sync(kFull, sd, pos);
        const uint32_t ti = __shfl_sync(kFull, sid, i);
        const uint32_t yi = __shfl_sync(kFull, sid, pos);
        if (t != y) {
          if (lane == i) { sd = y; sid = yi; }
          if (lane == pos) { sd = t; sid = ti; }
        }
      }
    }
    const unsigned val = __ballot_sync(kFull, !(sid & kVisited));
    const int x = val ? __ffs(val) - 1 : 32;
    if (x >= kNavBest) break;
    idx = x;
  }
  return static_cast<int>(__shfl_sync(kFull, sid, 0) & 0x7fffffffu);
}

// ADC table of one query into `lut` [M x 256] (shared or global memory).
// Lane l owns pivots 8l..8l+7 (two float4 loads per dimension). `qc` is q - c
// for L2 and q for the inner product.
template <bool IP>
__device__ __forceinline__ void build_lut(const DeviceIndex& ix, const float* __restrict__ qc,
                                          float* __restrict__ lut, int lane) {
  for (int c = 0; c < ix.chunks; ++c) {
    const int a0 = __ldg(ix.chunk_off + c), a1 = __ldg(ix.chunk_off + c + 1);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    for (int i = a0; i < a1; ++i) {
      const float qi = qc[i];
      const float4* p = reinterpret_cast<const float4*>(ix.pivots_t + static_cast<size_t>(i) * kPivots) + 2 * lane;
      const float4 p0 = __ldg(p), p1 = __ldg(p + 1);
      const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = dist_acc<IP>(qi, pv[k], acc[k]);
    }
    if (IP) {
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = -acc[k];
    }
    float4* o = reinterpret_cast<float4*>(lut + c * kPivots) + 2 * lane;
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// Sum LUT entries for up to 16 codes packed in `c`, in chunk order.
__device__ __forceinline__ float adc16(float s, const uint4 c, const float* __restrict__ lut, int n) {
  const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    if (b < n) s = __fadd_rn(s, lut[b * kPivots + ((w[b >> 2] >> (8 * (b & 3))) & 0xffu)]);
  }
  return s;
}

// CTA-resident PQ pivot table, row r = chunk * 256 + code. With 3 dims per
// chunk the rows are split into an (x, y) float2 plane and a z float plane:
// 12 B per pivot, gathered with one 8-byte and one 4-byte shared load, which
// costs fewer bank-conflict wavefronts for 32 random rows than one padded
// 16-byte row (about 9.0 against 10.2). Chunks of up to 4 dims keep float4
// rows, zero-padded.
struct PivTab {
  const float2* xy;
  const float* z;
  const float4* xyzw;
};

__host__ __device__ inline size_t piv_tab_bytes(int cw, int chunks) {
  return static_cast<size_t>(cw == 3 ? 12 : 16) * chunks * kPivots;
}

// The same sums without a per-query table: the table entry of chunk `b` and
// code `j` is recomputed from the pivot row of (b, j) and the query residual
// qcp[b] -- d = qc_i - p_ji, e = fma(d, d, e) from 0 over the chunk's dims in
// order, then s += e -- which are the fp32 operations that produce and consume
// the reference's table entry, so the sum is bit-identical. CW = dims per
// chunk (4 also serves mixed widths <= 4: the zero padding contributes
// fma(0, 0, e) = e). `row0` is the first row of this 16-chunk group.
template <int CW, bool IP>
__device__ __forceinline__ float adc16_piv(float s, const uint4 c, const PivTab& t, int row0,
                                           const float4* __restrict__ qcp, int n) {
  const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    if (b < n) {
      const float4 q = qcp[b];
      const int r = row0 + b * kPivots + static_cast<int>(__byte_perm(w[b >> 2], 0u, 0x4440u | (b & 3)));
      float4 p;
      if (CW == 3) {
        const float2 xy = t.xy[r];
        p = make_float4(xy.x, xy.y, t.z[r], 0.f);
      } else {
        p = t.xyzw[r];
      }
      if (IP) {
        // inner product: e = fma chain of q_i * p_ji from 0; entry = -e, and
        // s + (-e) is s - e
        float e = __fmaf_rn(q.x, p.x, 0.f);
        e = __fmaf_rn(q.y, p.y, e);
        e = __fmaf_rn(q.z, p.z, e);
        if (CW > 3) e = __fmaf_rn(q.w, p.w, e);
        s = __fsub_rn(s, e);
        continue;
      }
      // the x and y differences in one packed instruction (two independent
      // round-to-nearest subtractions, as __fsub_rn would give)
      float dx, dy;
      asm("{.reg .b64 a, b, c;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
          "sub.rn.f32x2 c, a, b;\n\tmov.b64 {%0, %1}, c;}"
          : "=f"(dx), "=f"(dy) : "f"(q.x), "f"(q.y), "f"(p.x), "f"(p.y));
      float e = __fmul_rn(dx, dx);
      e = __fmaf_rn(dy, dy, e);
      float d = __fsub_rn(q.z, p.z);
      e = __fmaf_rn(d, d, e);
      if (CW > 3) {
        d = __fsub_rn(q.w, p.w);
        e = __fmaf_rn(d, d, e);
      }
      s = __fadd_rn(s, e);
    }
  }
  return s;
}

// Table entry of chunk b for pivot row p: the reference's fp32 operations on
// the chunk's residual dims (as adc16_piv); CW = 3 when every chunk has 3
// dims, else 4 (zero padding contributes fma(0, 0, e) = e).
template <int CW>
__device__ __forceinline__ float piv_entry(const float4 q, const float4 p) {
  float dx, dy;
  asm("{.reg .b64 a, b, c;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "sub.rn.f32x2 c, a, b;\n\tmov.b64 {%0, %1}, c;}"
      : "=f"(dx), "=f"(dy) : "f"(q.x), "f"(q.y), "f"(p.x), "f"(p.y));
  float e = __fmul_rn(dx, dx);
  e = __fmaf_rn(dy, dy, e);
  float d = __fsub_rn(q.z, p.z);
  e = __fmaf_rn(d, d, e);
  if (CW > 3) {
    d = __fsub_rn(q.w, p.w);
    e = __fmaf_rn(d, d, e);
  }
  return e;
}

// Filtered mode: a per-query table of 8-bit lower bounds of the ADC table
// entries, lb(b, j) = mn_b + q_bj * sc <= entry(b, j) (real arithmetic), so
// that sum_b lb(b, code_b) = MN + sc * Q bounds the real sum of the entries of
// a candidate from below with one integer Q; the reference's sequential fp32
// sum of M non-negative entries is at least (1 - (M - 1) 2^-24) times the real
// sum, which kLbSlack covers for M <= 128. A candidate whose bound exceeds a
// full pool's last distance is cut by the reference's merge whatever its exact
// value, so its exact ADC is not needed.
constexpr float kLbSlack = 0.99999237060546875f;   // 1 - 2^-17
struct FiltParams {
  float sc = 1.f;       // quantisation step
  float mnsum = 0.f;    // sum of the per-chunk minima, rounded down
  float4 q = {0.f, 0.f, 0.f, 0.f};  // this lane's chunk residual (lane b = chunk b)
};

__device__ __forceinline__ float key_dist(uint64_t key) {
  const uint32_t b = static_cast<uint32_t>(key >> 32);
  return __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
}

// Sum of a candidate's 8-bit bounds over chunks 0..M-1 (integer, exact).
__device__ __forceinline__ int lut8_sum(const uint8_t* __restrict__ lut8, const uint4 c0, const uint4 c1, int M) {
  const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  int q = 0;
  if (M == 32) {
#pragma unroll
    for (int b = 0; b < 32; ++b) q += lut8[b * kPivots + static_cast<int>(__byte_perm(w[b >> 2], 0u, 0x4440u | (b & 3)))];
  } else {
#pragma unroll
    for (int b = 0; b < 32; ++b)
      if (b < M) q += lut8[b * kPivots + static_cast<int>(__byte_perm(w[b >> 2], 0u, 0x4440u | (b & 3)))];
  }
  return q;
}

// Build the 8-bit bound table of one query from q - c (`qc`, shared memory)
// and the pivot rows in global memory. The scale comes from chunk 0's range;
// any positive scale keeps the bounds valid, as entries above 255 steps clamp
// (a looser bound). A step is (entry - mn) / sc evaluated with every operation
// rounded toward zero on non-negative values, so it never exceeds the real
// quotient, and its integer part q satisfies mn + q * sc <= entry exactly.
template <int CW>
__device__ void build_lut8(const DeviceIndex& ix, const float* __restrict__ qc, uint8_t* __restrict__ lut8, int lane,
                           FiltParams& fp) {
  float sc = 1.f, inv = 1.f, mnsum = 0.f;   // inv <= 1 / sc
  for (int b = 0; b < ix.chunks; ++b) {
    const int a0 = __ldg(ix.chunk_off + b), a1 = __ldg(ix.chunk_off + b + 1);
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = a0 + i < a1 ? qc[a0 + i] : 0.f;
    const float4 q = make_float4(r[0], r[1], r[2], r[3]);
    float e[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) e[t] = piv_entry<CW>(q, __ldg(ix.piv4 + b * kPivots + lane + kWarp * t));
    float lo = e[0], hi = e[0];
#pragma unroll
    for (int t = 1; t < 8; ++t) {
      lo = fminf(lo, e[t]);
      hi = fmaxf(hi, e[t]);
    }
    // entries are >= +0, so their bit patterns order like the values
    const float mn = __uint_as_float(__reduce_min_sync(kFull, __float_as_uint(lo)));
    if (b == 0) {
      const float mx = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(hi)));
      sc = mx > mn ? __fmul_ru(__fsub_ru(mx, mn), 1.f / 255.f) : 1.f;
      inv = __frcp_rz(sc);
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float x = __fmul_rz(__fsub_rz(e[t], mn), inv);
      lut8[b * kPivots + lane + kWarp * t] = static_cast<uint8_t>(x >= 255.f ? 255 : static_cast<int>(x));
    }
    mnsum = __fadd_rd(mnsum, mn);
  }
  fp.sc = sc;
  fp.mnsum = mnsum;
}

struct WarpSmem {
  float* lut;     // per-query ADC table (table mode)
  float4* qcp;    // per-chunk query residuals, 4 dims padded (pivot mode)
  uint8_t* lut8;  // per-query 8-bit lower-bound table [M x 256] (filtered mode)
  float* ex;      // table entries of up to 8 candidates [8 x kExRow] (filtered mode)
  const uint8_t** xrow;  // code rows of the candidates whose exact ADC runs (filtered mode)
  float* xd;      // their exact ADC sums (filtered mode)
  float* qs;      // q, then q'' = (q - c) + c once the entry is known
  float* qc;      // q - c
  uint64_t* pool;  // up to ef keys, sorted
  uint64_t* cand;  // survivors' keys (merge)
  int* candr;      // survivors' pool ranks (merge); compacted neighbour ids at hop start
  int* hist;       // survivor ranks in key order (merge); compacted neighbour slots at hop start
  float* topd;     // top-k exact distances
  int* topi;       // top-k ids
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// Row stride (floats) of the filtered mode's entry matrix: 16-byte aligned
// rows that start 16 bytes apart in the banks, so 8 lanes reading a row each
// with 16-byte loads do not conflict.
constexpr int kExRow = 36;
constexpr int kExGroup = 8;   // candidates whose entries are computed together

enum CarveMode { kCarveTable = 0, kCarvePivot = 1, kCarveFilt = 2 };

// Shared-memory carve-up of one warp; mirrored by search_smem_bytes().
__host__ __device__ inline size_t carve(unsigned char* base, int chunks, int dim, int npl, int pl,
                                        int topk, WarpSmem* w, int mode = kCarveTable) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = base ? base + off : nullptr;
    off += align16(bytes);
    return p;
  };
  const int dpad = (dim + 3) & ~3;
  unsigned char* lut = mode == kCarveTable ? take(sizeof(float) * chunks * kPivots) : nullptr;
  unsigned char* qcp = mode == kCarvePivot ? take(sizeof(float4) * chunks) : nullptr;
  unsigned char *lut8 = nullptr, *ex = nullptr, *xrow = nullptr, *xd = nullptr;
  unsigned char *qs, *qc, *cand, *candr, *hist;
  const size_t a_q = align16(sizeof(float) * dpad);
  const size_t a_c = align16(sizeof(uint64_t) * npl * kWarp), a_r = align16(sizeof(int) * npl * kWarp);
  if (mode != kCarveFilt) {
    // query setup (qs, qc) and the hop buffers (cand, candr, hist) are never
    // live at once in a warp: qs is read into registers before the first hop
    unsigned char* reg = take(2 * a_q > a_c + 2 * a_r ? 2 * a_q : a_c + 2 * a_r);
    qs = reg;
    qc = reg ? reg + a_q : nullptr;
    cand = reg;
    candr = reg ? reg + a_c : nullptr;
    hist = reg ? reg + a_c + a_r : nullptr;
  } else {
    // the filtered mode's phases never overlap within a warp, so one region
    // holds in turn the query (setup: qs, qc), a hop's compacted neighbours
    // (candr, hist), the exact-ADC staging (ex, xrow, xd) and the merge
    // buffers (cand, candr, hist); __syncwarp separates the phases
    lut8 = take(static_cast<size_t>(chunks) * kPivots);
    const size_t a_ex = align16(sizeof(float) * kExGroup * kExRow), a_xr = align16(sizeof(void*) * npl * kWarp);
    const size_t a_xd = align16(sizeof(float) * npl * kWarp);
    size_t bytes = a_ex + a_xr + a_xd;
    bytes = bytes > 2 * a_q ? bytes : 2 * a_q;
    bytes = bytes > a_c + 2 * a_r ? bytes : a_c + 2 * a_r;
    unsigned char* reg = take(bytes);
    ex = reg;
    xrow = reg ? reg + a_ex : nullptr;
    xd = reg ? reg + a_ex + a_xr : nullptr;
    qs = reg;
    qc = reg ? reg + a_q : nullptr;
    cand = reg;
    candr = reg ? reg + a_c : nullptr;
    hist = reg ? reg + a_c + a_r : nullptr;
  }
  unsigned char* pool = take(sizeof(uint64_t) * pl * kWarp);
  unsigned char* topd = take(sizeof(float) * topk);
  unsigned char* topi = take(sizeof(int) * topk);
  if (w) {
    w->lut = reinterpret_cast<float*>(lut);
    w->qcp = reinterpret_cast<float4*>(qcp);
    w->lut8 = lut8;
    w->ex = reinterpret_cast<float*>(ex);
    w->xrow = reinterpret_cast<const uint8_t**>(xrow);
    w->xd = reinterpret_cast<float*>(xd);
    w->qs = reinterpret_cast<float*>(qs);
    w->qc = reinterpret_cast<float*>(qc);
    w->pool = reinterpret_cast<uint64_t*>(pool);
    w->cand = reinterpret_cast<uint64_t*>(cand);
    w->candr = reinterpret_cast<int*>(candr);
    w->hist = reinterpret_cast<int*>(hist);
    w->topd = reinterpret_cast<float*>(topd);
    w->topi = reinterpret_cast<int*>(topi);
  }
  return off;
}

// Addresses of node u's adjacency row, vector and neighbour-code block, in
// the single arrays or, with split records, in the arrays of u's part.
__device__ __forceinline__ const uint32_t* adj_row(const DeviceIndex& ix, uint32_t u) {
  if (ix.nparts > 1)
    return ix.part_adj[u >> ix.part_shift] +
           static_cast<size_t>(u & ((1u << ix.part_shift) - 1u)) * ix.adj_stride;
  return ix.adj + static_cast<size_t>(u) * ix.adj_stride;
}
__device__ __forceinline__ const uint8_t* vec_row(const DeviceIndex& ix, uint32_t u) {
  if (ix.nparts > 1)
    return ix.part_vecs[u >> ix.part_shift] +
           static_cast<size_t>(u & ((1u << ix.part_shift) - 1u)) * ix.vec_stride;
  return ix.vecs + static_cast<size_t>(u) * ix.vec_stride;
}
__device__ __forceinline__ const uint8_t* ncode_row(const DeviceIndex& ix, uint32_t u) {
  const size_t row = static_cast<size_t>(ix.adj_stride) * ix.code_stride;
  if (ix.nparts > 1)
    return ix.part_ncodes[u >> ix.part_shift] + static_cast<size_t>(u & ((1u << ix.part_shift) - 1u)) * row;
  return ix.ncodes + static_cast<size_t>(u) * row;
}

// Neighbour ids (padding = kPadId) and the vector elements lane l owns
// (dims l, l+32, ...) of one record. With the neighbour-code layout the node's
// block of neighbour code rows, whose address depends only on the node, is
// prefetched into L2 (no registers held while the merge runs; the hop that
// expands the node loads the rows it needs from L2) -- when the block is in
// this GPU's memory: an L2 prefetch of a peer GPU's address made split-record
// searches ~50x slower on B200, so remote blocks are simply loaded.
template <typename T, int NPL, int VP>
__device__ __forceinline__ void load_node(const DeviceIndex& ix, uint32_t u, int lane, uint32_t (&nb)[NPL],
                                          float (&xv)[VP]) {
  const uint32_t* arow = adj_row(ix, u);
#pragma unroll
  for (int k = 0; k < NPL; ++k) {
    const int e = lane + kWarp * k;
    nb[k] = e < ix.degree ? __ldg(arow + e) : kPadId;
  }
  const bool local = ix.nparts <= 1 || ix.local_part < 0 || static_cast<int>(u >> ix.part_shift) == ix.local_part;
  if (ix.ncodes != nullptr && local) {
    const uint8_t* crow = ncode_row(ix, u);
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const int e = lane + kWarp * k;
      if (e < ix.degree) asm volatile("prefetch.global.L2 [%0];" ::"l"(crow + static_cast<size_t>(e) * ix.code_stride));
    }
  }
  const T* xr = reinterpret_cast<const T*>(vec_row(ix, u));
#pragma unroll
  for (int v = 0; v < VP; ++v) {
    const int i = lane + kWarp * v;
    xv[v] = i < ix.dim ? static_cast<float>(__ldg(xr + i)) : 0.f;
  }
}

// Code gather for the neighbour-code layout: out row u, slot k = codes of
// adj[u][k] (zeros for empty slots). One thread per 16-byte word.
__global__ void gather_neighbour_codes(const uint32_t* __restrict__ adj, int adj_stride, int degree,
                                       const uint4* __restrict__ codes, int words, int64_t n, uint4* __restrict__ out) {
  const int64_t total = n * adj_stride * words;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t slot = i / words;
    const int w = static_cast<int>(i % words);
    const int k = static_cast<int>(slot % adj_stride);
    const uint32_t v = k < degree ? __ldg(adj + slot) : kPadId;
    out[i] = v != kPadId ? __ldg(codes + static_cast<int64_t>(v) * words + w) : make_uint4(0, 0, 0, 0);
  }
}

// Best-first traversal of one query from `entry` (src/impl/pure_mem.cuh:285-428).
//
// The node expanded next is min(first unvisited pool entry, best candidate
// that enters the pool) -- exactly the first unvisited entry of the merged
// pool -- so it is known right after the ADC step. Its record is requested
// then (adjacency and vector into registers, neighbour code rows into L2), and
// the merge and the top-k insert of the current node run while those loads are
// in flight.
//
// Neighbours whose ADC cannot change the pool are skipped: the warp's visited
// table (2^kVisBits ids in global memory, L2-resident, cleared per query) is a
// lossy direct-mapped set of the ids evaluated earlier in this query, never
// wrong in that direction. Such a node is either in the pool (a duplicate of
// the pool copy, same id and distance) or was dropped or pushed out while the
// pool was full; a full pool's last key never grows, so it would be dropped
// again. The remaining neighbours are compacted to the low lanes, so a hop
// with at most 32 of them runs one ADC pass instead of NPL. (Without a table,
// e.g. gann_search_noalloc, every neighbour is evaluated; duplicates of pool
// entries are then dropped by the rank search.)
template <typename T, int NPL, int VP, int PIV, bool IP, bool FILT>
__device__ void traverse(const DeviceIndex& ix, const SearchArgs& a, int64_t qid, uint32_t entry,
                         const WarpSmem& s, const PivTab& piv, int lane, int pl, const FiltParams& fp) {
  const int dim = ix.dim, M = ix.chunks, L = a.ef, topk = a.topk;
  const int mw = ix.code_stride >> 4;
  int psize = 0, tcnt = 0, pfirst = 0;
  uint32_t hops = 0, adc = 0;
  uint32_t u = entry;
  bool capped = false;

  // this warp's visited table (none when the caller gave no buffer)
  const int64_t wslot = static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarp) + threadIdx.x / kWarp;
  uint32_t* const vis = a.vis != nullptr && wslot < a.vis_slots ? a.vis + (wslot << kVisBits) : nullptr;
  auto vslot = [](uint32_t id) { return static_cast<int>((id * 0x9E3779B1u) >> (32 - kVisBits)); };
  if (vis != nullptr)
    for (int i = 4 * lane; i < (1 << kVisBits); i += 4 * kWarp)
      *reinterpret_cast<uint4*>(vis + i) = make_uint4(kPadId, kPadId, kPadId, kPadId);
  float qv[VP];   // q'' = (q - c) + c (q for the inner product), the lane's dims
#pragma unroll
  for (int v = 0; v < VP; ++v) {
    const int i = lane + kWarp * v;
    qv[v] = i < dim ? s.qs[i] : 0.f;
  }
  uint32_t nb[NPL];
  float xv[VP];
  load_node<T, NPL, VP>(ix, u, lane, nb, xv);
  __syncwarp();
  int ppos = -1;            // the pool is empty before the first hop
  uint64_t pstar = ~0ull;

  for (;;) {
    if (hops >= static_cast<uint32_t>(a.max_hops)) {
      capped = true;
      break;
    }
    ++hops;
    // neighbours to evaluate, compacted to lanes 0.. of pass 0, then pass 1
    // (ids in candr, neighbour slots in hist until the merge reuses both)
    uint32_t seen[NPL];
#pragma unroll
    for (int k = 0; k < NPL; ++k) seen[k] = vis != nullptr && nb[k] != kPadId ? vis[vslot(nb[k])] : kPadId;
    int cnt = 0;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      adc += __popc(__ballot_sync(kFull, nb[k] != kPadId));
      const bool e = nb[k] != kPadId && seen[k] != nb[k];
      const unsigned bm = __ballot_sync(kFull, e);
      if (e) {
        const int pos = cnt + __popc(bm & ((1u << lane) - 1u));
        s.candr[pos] = static_cast<int>(nb[k]);
        s.hist[pos] = lane + kWarp * k;
      }
      cnt += __popc(bm);
    }
    __syncwarp();
    // their code rows: slot of u's neighbour-code block (prefetched into L2
    // when u was chosen), else row id of `codes`; ids enter the visited table
    bool ok[NPL];
    const uint4* crow[NPL];
    uint4 c0[NPL], c1[NPL];
    const bool inl = ix.ncodes != nullptr;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const int j = lane + kWarp * k;
      ok[k] = j < cnt;
      nb[k] = ok[k] ? static_cast<uint32_t>(s.candr[j]) : kPadId;
      const int slot = ok[k] ? s.hist[j] : 0;
      crow[k] = reinterpret_cast<const uint4*>(
          inl ? ncode_row(ix, u) + static_cast<size_t>(slot) * ix.code_stride
              : ix.codes + static_cast<size_t>(ok[k] ? nb[k] : 0) * ix.code_stride);
      c0[k] = ok[k] ? __ldg(crow[k]) : make_uint4(0, 0, 0, 0);
      c1[k] = (ok[k] && mw > 1) ? __ldg(crow[k] + 1) : make_uint4(0, 0, 0, 0);
      if (ok[k] && vis != nullptr) vis[vslot(nb[k])] = nb[k];
    }
    __syncwarp();

    // pstar = the first unvisited pool entry, at ppos (found at the end of
    // the previous hop)

    // ADC of every neighbour not known to be in the pool, chunks in order
    float dsum[NPL];
#pragma unroll
    for (int k = 0; k < NPL; ++k) dsum[k] = 0.f;
    if constexpr (FILT) {
      // a full pool: candidates whose 8-bit bound exceeds its last distance
      // are dropped without their exact ADC
      if (psize == L) {
        const float lastd = key_dist(s.pool[L - 1]);
        // first slot: one lane per candidate, 32 byte lookups each
        if (__any_sync(kFull, ok[0])) {
          const int qsum = lut8_sum(s.lut8, c0[0], c1[0], M);
          const float lb = __fmaf_rd(fp.sc, static_cast<float>(qsum), fp.mnsum);
          if (ok[0] && __fmul_rd(lb, kLbSlack) > lastd) ok[0] = false;
        }
        // later slots hold few candidates: the warp sums each one's bounds,
        // lane b looking up chunk b (integer sums, exact in any order)
#pragma unroll
        for (int k = 1; k < NPL; ++k) {
          for (unsigned m = __ballot_sync(kFull, ok[k]); m; m &= m - 1) {
            const int src = __ffs(m) - 1;
            const uint8_t* row = reinterpret_cast<const uint8_t*>(
                __shfl_sync(kFull, reinterpret_cast<unsigned long long>(crow[k]), src));
            const unsigned v = lane < M ? s.lut8[lane * kPivots + __ldg(row + lane)] : 0u;
            const unsigned qsum = __reduce_add_sync(kFull, v);
            const float lb = __fmaf_rd(fp.sc, static_cast<float>(qsum), fp.mnsum);
            if (lane == src && __fmul_rd(lb, kLbSlack) > lastd) ok[k] = false;
          }
        }
      }
      // exact ADC of the rest: lane b computes chunk b's table entry of up to
      // kExGroup candidates (the reference's fp32 operations on the pivot row),
      // then one lane per candidate adds the entries in chunk order
      int xpos[NPL];
      int nx = 0;
#pragma unroll
      for (int k = 0; k < NPL; ++k) {
        const unsigned bm = __ballot_sync(kFull, ok[k]);
        xpos[k] = nx + __popc(bm & ((1u << lane) - 1u));
        if (ok[k]) s.xrow[xpos[k]] = reinterpret_cast<const uint8_t*>(crow[k]);
        nx += __popc(bm);
      }
      __syncwarp();
      for (int g = 0; g < nx; g += kExGroup) {
        const int gn = min(kExGroup, nx - g);
        float4 pr[kExGroup];
#pragma unroll
        for (int c = 0; c < kExGroup; ++c) {
          pr[c] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (c < gn && lane < M) pr[c] = __ldg(ix.piv4 + lane * kPivots + __ldg(s.xrow[g + c] + lane));
        }
#pragma unroll
        for (int c = 0; c < kExGroup; ++c)
          if (c < gn && lane < M) s.ex[c * kExRow + lane] = piv_entry<PIV>(fp.q, pr[c]);
        __syncwarp();
        if (lane < gn) {
          const float4* row = reinterpret_cast<const float4*>(s.ex + lane * kExRow);
          float acc = 0.f;
          if (M == 32) {
#pragma unroll
            for (int b4 = 0; b4 < 8; ++b4) {
              const float4 e = row[b4];
              acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, e.x), e.y), e.z), e.w);
            }
          } else {
            for (int b = 0; b < M; ++b) acc = __fadd_rn(acc, s.ex[lane * kExRow + b]);
          }
          s.xd[g + lane] = acc;
        }
        __syncwarp();
      }
#pragma unroll
      for (int k = 0; k < NPL; ++k)
        if (ok[k]) dsum[k] = s.xd[xpos[k]];
    } else for (int w = 0; w < mw; ++w) {
      uint4 cur[NPL];
#pragma unroll
      for (int k = 0; k < NPL; ++k)
        cur[k] = w == 0 ? c0[k] : w == 1 ? c1[k] : (ok[k] ? __ldg(crow[k] + w) : make_uint4(0, 0, 0, 0));
      const int n = min(16, M - 16 * w);
      if (PIV == 0) {
        const float* lw = s.lut + 16 * w * kPivots;
#pragma unroll
        for (int k = 0; k < NPL; ++k)
          if (ok[k]) dsum[k] = adc16(dsum[k], cur[k], lw, n);
      } else if (n == 16) {
        // a full word: the chunk bound folds away (the common case, M % 16 == 0)
        const float4* qw = s.qcp + 16 * w;
#pragma unroll
        for (int k = 0; k < NPL; ++k)
          if (ok[k]) dsum[k] = PIV == 3 ? adc16_piv<3, IP>(dsum[k], cur[k], piv, 16 * w * kPivots, qw, 16)
                                        : adc16_piv<4, IP>(dsum[k], cur[k], piv, 16 * w * kPivots, qw, 16);
      } else {
        const float4* qw = s.qcp + 16 * w;
#pragma unroll
        for (int k = 0; k < NPL; ++k)
          if (ok[k]) dsum[k] = PIV == 3 ? adc16_piv<3, IP>(dsum[k], cur[k], piv, 16 * w * kPivots, qw, n)
                                        : adc16_piv<4, IP>(dsum[k], cur[k], piv, 16 * w * kPivots, qw, n);
      }
    }

    // candidates that can enter the pool: not beyond its last entry when full,
    // not already in it; rank = insertion point (lower bound on (dist, id)),
    // found by power-of-two steps with a warp-uniform trip count and the NPL
    // searches of a lane interleaved (independent shared loads in flight)
    uint64_t key[NPL];
    int rk[NPL];
    const uint64_t last = psize == L ? (s.pool[L - 1] >> 1) : ~0ull;
    uint64_t mk = ~0ull;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      key[k] = make_key(dsum[k], nb[k]);
      rk[k] = 0;
      if (ok[k] && (key[k] >> 1) >= last) ok[k] = false;
    }
    // slots past the first only need a search when a lane still holds a live
    // candidate there (after the drops above, rarely once the pool is full)
    bool multi = false;
#pragma unroll
    for (int k = 1; k < NPL; ++k) multi = multi || __any_sync(kFull, ok[k]);
    if (psize > 0 && multi) {
      for (int step = 1 << (31 - __clz(psize)); step > 0; step >>= 1) {
#pragma unroll
        for (int k = 0; k < NPL; ++k) {
          const int t = rk[k] + step;
          if (ok[k] && t <= psize && (s.pool[t - 1] >> 1) < (key[k] >> 1)) rk[k] = t;
        }
      }
    } else if (psize > 0) {
      // only the first slot holds live candidates
      for (int step = 1 << (31 - __clz(psize)); step > 0; step >>= 1) {
        const int t = rk[0] + step;
        if (ok[0] && t <= psize && (s.pool[t - 1] >> 1) < (key[0] >> 1)) rk[0] = t;
      }
    }
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      if (ok[k] && rk[k] < psize && (s.pool[rk[k]] >> 1) == (key[k] >> 1)) ok[k] = false;
      if (ok[k] && key[k] < mk) mk = key[k];
    }
    {
      // warp minimum of the 64-bit keys: the high words, then the low words of
      // the lanes holding that high word (two redux.sync instead of 5 shuffle rounds)
      const uint32_t mhi = __reduce_min_sync(kFull, static_cast<uint32_t>(mk >> 32));
      const uint32_t mlo = __reduce_min_sync(kFull, static_cast<uint32_t>(mk >> 32) == mhi
                                                        ? static_cast<uint32_t>(mk) : 0xffffffffu);
      mk = (static_cast<uint64_t>(mhi) << 32) | mlo;
    }
    const uint64_t nxt = mk < pstar ? mk : pstar;
    const bool more = nxt != ~0ull;
    uint32_t nb2[NPL];
    float xv2[VP];
    if (more) {
      load_node<T, NPL, VP>(ix, static_cast<uint32_t>(nxt) >> 1, lane, nb2, xv2);
    } else {
#pragma unroll
      for (int k = 0; k < NPL; ++k) nb2[k] = kPadId;
#pragma unroll
      for (int v = 0; v < VP; ++v) xv2[v] = 0.f;
    }

    // exact distance of u (lane-strided fma, shfl_down tree), then insert after
    // every equal entry of the top-k (retset_push_32, src/impl/util.cuh:116-163)
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < VP; ++v) {
      if (lane + kWarp * v < dim) acc = dist_acc<IP>(qv[v], xv[v], acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, off));
    const float ex = IP ? -__shfl_sync(kFull, acc, 0) : __shfl_sync(kFull, acc, 0);
    {
      int le = 0;
      for (int t0 = 0; t0 < tcnt; t0 += kWarp) {
        const int t = t0 + lane;
        le += __popc(__ballot_sync(kFull, t < tcnt && s.topd[t] <= ex));
      }
      if (le < topk) {
        const int hi = min(tcnt, topk - 1);
        if (hi > le) {
          const int nch = (hi - le + kWarp - 1) / kWarp;
          for (int c = nch - 1; c >= 0; --c) {
            const int t = le + c * kWarp + lane;
            const bool v = t < hi;
            float dv = 0.f;
            int iv = 0;
            if (v) { dv = s.topd[t]; iv = s.topi[t]; }
            __syncwarp();
            if (v) { s.topd[t + 1] = dv; s.topi[t + 1] = iv; }
            __syncwarp();
          }
        }
        if (lane == 0) {
          s.topd[le] = ex;
          s.topi[le] = static_cast<int>(u);
        }
      }
      tcnt = min(tcnt + 1, topk);
    }

    // merge the surviving candidates into the pool; the entry equal to `nxt`
    // is written back marked visited
    int S = 0;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const unsigned bm = __ballot_sync(kFull, ok[k]);
      if (ok[k]) {
        const int slot = S + __popc(bm & ((1u << lane) - 1u));
        s.cand[slot] = key[k];
        s.candr[slot] = rk[k];
      }
      S += __popc(bm);
    }
    __syncwarp();
    if (S > 0) {
      // final slot of each survivor = rank in pool + rank among survivors
      uint64_t ck[NPL];
      int cpos[NPL], cr[NPL];
      int rmin = INT_MAX;
#pragma unroll
      for (int k = 0; k < NPL; ++k) {
        const int si = lane + kWarp * k;
        cpos[k] = INT_MAX;
        cr[k] = 0;
        ck[k] = 0;
        if (si < S) {
          ck[k] = s.cand[si];
          cr[k] = s.candr[si];
          const uint64_t kk = ck[k] >> 1;
          int less = 0;
          for (int t = 0; t < S; ++t) {
            const uint64_t o = s.cand[t] >> 1;
            less += (o < kk) || (o == kk && t < si);
          }
          cpos[k] = cr[k] + less;
          if (ck[k] == nxt) ck[k] &= ~1ull;
          rmin = min(rmin, cr[k]);
        }
      }
      int rmax = 0;
#pragma unroll
      for (int k = 0; k < NPL; ++k)
        if (lane + kWarp * k < S) rmax = max(rmax, cr[k]);
      rmin = __reduce_min_sync(kFull, rmin);
      rmax = static_cast<int>(__reduce_max_sync(kFull, static_cast<unsigned>(rmax)));
      // survivor ranks in key order are non-decreasing: hist[t] = rank of the
      // t-th smallest survivor; entry i >= rmin moves right by #{t : hist[t] <= i}
#pragma unroll
      for (int k = 0; k < NPL; ++k)
        if (lane + kWarp * k < S) s.hist[cpos[k] - cr[k]] = cr[k];
      __syncwarp();
      // moves, from the last chunk down (an entry only moves right); entries
      // pushed past `ef` leave the pool. Chunks at or after the largest
      // survivor rank move by S as a whole (every survivor ranks before them);
      // the chunks from rmin up to there take each entry's shift, an upper bound
      // in hist, found by power-of-two steps with four chunks interleaved.
      const int j0 = rmin >> 5;
      const int ju = (rmax + kWarp - 1) >> 5;
      for (int j = min((psize - 1) >> 5, (L - 1 - S) >> 5); j >= ju && j >= j0; --j) {
        const int i = lane + kWarp * j;
        uint64_t v = i < psize ? s.pool[i] : 0;
        if (v == nxt) v &= ~1ull;
        __syncwarp();
        if (i < psize && i + S < L) s.pool[i + S] = v;
      }
      __syncwarp();
      const int sstep = 1 << (31 - __clz(S));
      for (int jg = min((psize - 1) >> 5, ju - 1); jg >= j0; jg -= 4) {
        uint64_t v[4];
        int dst[4], sh[4];
        bool act[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int i = lane + kWarp * (jg - g);
          act[g] = jg - g >= j0 && i < psize;
          v[g] = act[g] ? s.pool[i] : 0;
          sh[g] = 0;
        }
        for (int step = sstep; step > 0; step >>= 1) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int t = sh[g] + step;
            if (act[g] && t <= S && s.hist[t - 1] <= lane + kWarp * (jg - g)) sh[g] = t;
          }
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          dst[g] = act[g] ? lane + kWarp * (jg - g) + sh[g] : INT_MAX;
          if (v[g] == nxt) v[g] &= ~1ull;
        }
        __syncwarp();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (dst[g] < L) {
            s.pool[dst[g]] = v[g];
          }
        }
        __syncwarp();
      }
#pragma unroll
      for (int k = 0; k < NPL; ++k) {
        if (cpos[k] < L) {
          s.pool[cpos[k]] = ck[k];
        }
      }
      // a next node taken from the pool in front of every survivor keeps its
      // slot and was not rewritten by the moves above: mark it here
      if (nxt == pstar && ppos < kWarp * j0 && lane == 0) s.pool[ppos] = pstar & ~1ull;
      psize = min(psize + S, L);
      pfirst = min(pfirst, rmin);
    } else if (more && lane == 0) {
      s.pool[ppos] = pstar & ~1ull;   // no survivor: the next node is pool entry ppos
    }
    __syncwarp();
    if (!more) break;
    u = static_cast<uint32_t>(nxt) >> 1;
#pragma unroll
    for (int k = 0; k < NPL; ++k) nb[k] = nb2[k];
#pragma unroll
    for (int v = 0; v < VP; ++v) xv[v] = xv2[v];

    // first unvisited pool entry for the next hop (every entry before
    // `pfirst` is visited); scanned here, while the next node's record loads
    // are in flight, rather than after the next hop's visited-table reads
    ppos = -1;
    for (int j = pfirst >> 5; kWarp * j < psize; ++j) {
      const int i = lane + kWarp * j;
      const unsigned bm = __ballot_sync(kFull, i < psize && (s.pool[i] & 1ull));
      if (bm) {
        ppos = kWarp * j + __ffs(bm) - 1;
        break;
      }
    }
    pfirst = ppos >= 0 ? ppos : psize;
    pstar = ppos >= 0 ? s.pool[ppos] : ~0ull;
  }

  int32_t* nns = a.nns + qid * topk;
  float* dist = a.dist + qid * topk;
  for (int t = lane; t < topk; t += kWarp) {
    const bool v = t < tcnt;
    nns[t] = v ? s.topi[t] : 0;
    dist[t] = v ? s.topd[t] : 0.f;
  }
  if (lane == 0) {
    a.found[qid] = tcnt;
    if (a.hops) a.hops[qid] = hops;
    if (a.adc) a.adc[qid] = adc;
    if (capped) atomicAdd(a.err, 1);
  }
}

// One query per warp, from query setup to the written top-k.
template <typename T, int NPL, int VP, int PIV, bool IP, bool FILT = false>
__device__ __forceinline__ void run_queries(const DeviceIndex& ix, const SearchArgs& a, const WarpSmem& s,
                                            const PivTab& piv, int lane, int pl) {
  const int dim = ix.dim;
  for (;;) {
    int qid = 0;
    if (lane == 0) qid = atomicAdd(a.qcounter, 1);
    qid = __shfl_sync(kFull, qid, 0);
    if (qid >= a.nq) break;
    const float* q = a.q + static_cast<int64_t>(qid) * dim;
    for (int i = lane; i < dim; i += kWarp) {
      const float v = q[i];
      s.qs[i] = v;
      s.qc[i] = __fsub_rn(v, __ldg(ix.centroid + i));
    }
    __syncwarp();
    uint32_t entry = static_cast<uint32_t>(ix.medoid);
    if (ix.has_nav) {
      bool capped = false;
      const int si = nav_search<T, IP>(ix, s.qs, lane, a.nav_max_hops, capped);
      // slot 0 can end up holding an empty slot on degenerate graphs (a node
      // whose only neighbour is itself); the reference then indexes its map out
      // of range, here the query falls back to the medoid and is counted
      const bool bad = si < 0 || si >= ix.nav_points;
      if (!bad) entry = static_cast<uint32_t>(__ldg(ix.nav_map + si));
      if ((capped || bad) && lane == 0) atomicAdd(a.err + 1, 1);
    }
    __syncwarp();
    if (!IP)
      for (int i = lane; i < dim; i += kWarp) s.qs[i] = __fadd_rn(s.qc[i], __ldg(ix.centroid + i));
    // the table / pivot-mode query terms: q - c for L2, q for the inner product
    const float* qt = IP ? s.qs : s.qc;
    FiltParams fp;
    if constexpr (FILT) {
      // lane b keeps chunk b's residual dims; the 8-bit bound table
      if (lane < ix.chunks) {
        const int a0 = __ldg(ix.chunk_off + lane), a1 = __ldg(ix.chunk_off + lane + 1);
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = a0 + i < a1 ? qt[a0 + i] : 0.f;
        fp.q = make_float4(r[0], r[1], r[2], r[3]);
      }
      build_lut8<PIV>(ix, qt, s.lut8, lane, fp);
    } else if (PIV == 0) {
      build_lut<IP>(ix, qt, s.lut, lane);
    } else {
      for (int c = lane; c < ix.chunks; c += kWarp) {
        const int a0 = __ldg(ix.chunk_off + c), a1 = __ldg(ix.chunk_off + c + 1);
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = a0 + i < a1 ? qt[a0 + i] : 0.f;
        s.qcp[c] = make_float4(r[0], r[1], r[2], r[3]);
      }
    }
    __syncwarp();
    traverse<T, NPL, VP, PIV, IP, FILT>(ix, a, qid, entry, s, piv, lane, pl, fp);
    __syncwarp();
  }
}

// Table mode: one warp per CTA, the warp's ADC table in its shared memory.
template <typename T, int NPL, int VP, bool IP>
__global__ void __launch_bounds__(kWarp) search_kernel(const DeviceIndex ix, const SearchArgs a, int pl) {
  extern __shared__ __align__(16) unsigned char smem[];
  WarpSmem s;
  carve(smem, ix.chunks, ix.dim, NPL, pl, a.topk, &s, kCarveTable);
  run_queries<T, NPL, VP, 0, IP>(ix, a, s, PivTab{nullptr, nullptr, nullptr}, threadIdx.x, pl);
}

// Pivot mode: one persistent CTA per SM holds the 256 x D pivot table once
// (M x 3 KB for 3-dim chunks, M x 4 KB otherwise) and runs up to piv_warps_max
// queries at a time, one per warp, each with a few KB of private state instead
// of a 4*M KB table.
// Queries per SM: 24 at two neighbours per lane (80 registers a thread, no
// spills); 20 at four, whose extra registers would spill at 24.
constexpr int piv_warps_max(int npl) { return npl > 2 ? 20 : 24; }
template <typename T, int NPL, int VP, int CW, bool IP>
__global__ void __launch_bounds__(kWarp * piv_warps_max(NPL), 1) search_kernel_piv(const DeviceIndex ix, const SearchArgs a,
                                                                          size_t per_warp, int pl) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int ntab = ix.chunks * kPivots;
  PivTab piv{nullptr, nullptr, nullptr};
  if (CW == 3) {
    float2* xy = reinterpret_cast<float2*>(smem);
    float* z = reinterpret_cast<float*>(xy + ntab);
    for (int i = threadIdx.x; i < ntab; i += blockDim.x) {
      const float4 p = __ldg(ix.piv4 + i);
      xy[i] = make_float2(p.x, p.y);
      z[i] = p.z;
    }
    piv.xy = xy;
    piv.z = z;
  } else {
    float4* t = reinterpret_cast<float4*>(smem);
    for (int i = threadIdx.x; i < ntab; i += blockDim.x) t[i] = __ldg(ix.piv4 + i);
    piv.xyzw = t;
  }
  __syncthreads();
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  WarpSmem s;
  carve(smem + piv_tab_bytes(CW, ix.chunks) + per_warp * warp, ix.chunks, ix.dim, NPL, pl, a.topk, &s, kCarvePivot);
  run_queries<T, NPL, VP, CW, IP>(ix, a, s, piv, lane, pl);
}

// Filtered mode: no CTA-wide pivot table in shared memory; each warp keeps
// its query's 8-bit bound table (M x 256 B) and reads the pivot rows of the
// few candidates that need an exact ADC from global memory (L2-resident).
constexpr int kFiltWarpsMax = 20;
template <typename T, int NPL, int VP, int CW>
__global__ void __launch_bounds__(kWarp * kFiltWarpsMax, 1) search_kernel_filt(const DeviceIndex ix, const SearchArgs a,
                                                                               size_t per_warp, int pl) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  WarpSmem s;
  carve(smem + per_warp * warp, ix.chunks, ix.dim, NPL, pl, a.topk, &s, kCarveFilt);
  run_queries<T, NPL, VP, CW, false, true>(ix, a, s, PivTab{nullptr, nullptr, nullptr}, lane, pl);
}

template <bool IP>
__global__ void __launch_bounds__(kWarp) probe_lut_kernel(const DeviceIndex ix, const float* q, int64_t nq,
                                                          float* lut) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qc = reinterpret_cast<float*>(smem);
  const int lane = threadIdx.x;
  for (int64_t qid = blockIdx.x; qid < nq; qid += gridDim.x) {
    for (int i = lane; i < ix.dim; i += kWarp)
      qc[i] = IP ? q[qid * ix.dim + i] : __fsub_rn(q[qid * ix.dim + i], __ldg(ix.centroid + i));
    __syncwarp();
    build_lut<IP>(ix, qc, lut + qid * ix.chunks * kPivots, lane);
    __syncwarp();
  }
}

template <typename T, bool IP>
__global__ void __launch_bounds__(kWarp) probe_entry_kernel(const DeviceIndex ix, const float* q, int64_t nq,
                                                            int32_t* sample, int32_t* entry, int32_t* err,
                                                            int max_hops) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qs = reinterpret_cast<float*>(smem);
  const int lane = threadIdx.x;
  for (int64_t qid = blockIdx.x; qid < nq; qid += gridDim.x) {
    for (int i = lane; i < ix.dim; i += kWarp) qs[i] = q[qid * ix.dim + i];
    __syncwarp();
    bool capped = false;
    const int si = nav_search<T, IP>(ix, qs, lane, max_hops, capped);
    const bool bad = si < 0 || si >= ix.nav_points;
    if (lane == 0) {
      sample[qid] = si;
      entry[qid] = bad ? static_cast<int32_t>(ix.medoid) : __ldg(ix.nav_map + si);
      if (capped || bad) atomicAdd(err, 1);
    }
    __syncwarp();
  }
}

int npl_for(int degree) { return degree <= 64 ? 2 : 4; }
int pl_for(int ef) { return (ef + kWarp - 1) / kWarp; }
int vp_for(int dim) { return dim <= 128 ? 4 : 32; }

template <typename T, int NPL, int VP, bool IP>
cudaError_t launch_variant(const DeviceIndex& ix, const SearchArgs& a, int sm_count, cudaStream_t st) {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int pl = pl_for(a.ef);
  if constexpr (VP == 4 && !IP) if (ix.piv_width > 0 && ix.chunks <= kWarp && ix.adc_mode == 3) {
    // filtered mode: as many warps as their shared memory allows (<= 20)
    const size_t per_warp = carve(nullptr, ix.chunks, ix.dim, NPL, pl, a.topk, nullptr, kCarveFilt);
    int warps = static_cast<int>(std::min<size_t>(kFiltWarpsMax, optin / per_warp));
    if (ix.piv_warps > 0) warps = std::min(warps, ix.piv_warps);
    if (warps >= 8) {
      const size_t smem = per_warp * warps;
      auto fn = ix.piv_width == 3 ? search_kernel_filt<T, NPL, VP, 3> : search_kernel_filt<T, NPL, VP, 4>;
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      int64_t grid = std::min<int64_t>(sm_count, (a.nq + warps - 1) / warps);
      if (grid <= 0) return cudaSuccess;
      fn<<<static_cast<unsigned>(grid), kWarp * warps, smem, st>>>(ix, a, per_warp, pl);
      return cudaGetLastError();
    }
  }
  if constexpr (VP == 4) if (ix.piv_width > 0 && ix.adc_mode != 1) {
    // pivot mode when the table plus at least 8 warps' state fit (dims <= 128;
    // wider vectors have too many chunks for a shared-memory pivot table)
    const size_t tab = piv_tab_bytes(ix.piv_width, ix.chunks);
    const size_t per_warp = carve(nullptr, ix.chunks, ix.dim, NPL, pl, a.topk, nullptr, kCarvePivot);
    int warps = tab < static_cast<size_t>(optin)
                    ? static_cast<int>(std::min<size_t>(piv_warps_max(NPL), (optin - tab) / per_warp)) : 0;
    if (ix.piv_warps > 0) warps = std::min(warps, ix.piv_warps);
    if (warps >= 8) {
      const size_t smem = tab + per_warp * warps;
      auto fn = ix.piv_width == 3 ? search_kernel_piv<T, NPL, VP, 3, IP> : search_kernel_piv<T, NPL, VP, 4, IP>;
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      int64_t grid = std::min<int64_t>(sm_count, (a.nq + warps - 1) / warps);
      if (grid <= 0) return cudaSuccess;
      fn<<<static_cast<unsigned>(grid), kWarp * warps, smem, st>>>(ix, a, per_warp, pl);
      return cudaGetLastError();
    }
  }
  const size_t smem = carve(nullptr, ix.chunks, ix.dim, NPL, pl, a.topk, nullptr, kCarveTable);
  auto fn = search_kernel<T, NPL, VP, IP>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kWarp, smem);
  if (e != cudaSuccess) return e;
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  int64_t grid = static_cast<int64_t>(per_sm) * sm_count;
  if (grid > a.nq) grid = a.nq;
  if (grid <= 0) return cudaSuccess;
  fn<<<static_cast<unsigned>(grid), kWarp, smem, st>>>(ix, a, pl);
  return cudaGetLastError();
}

template <typename T, int VP>
cudaError_t launch_vp(const DeviceIndex& ix, const SearchArgs& a, int sm_count, cudaStream_t st) {
  const bool ip = ix.metric == GANN_METRIC_IP;
  if (npl_for(ix.degree) == 2)
    return ip ? launch_variant<T, 2, VP, true>(ix, a, sm_count, st) : launch_variant<T, 2, VP, false>(ix, a, sm_count, st);
  return ip ? launch_variant<T, 4, VP, true>(ix, a, sm_count, st) : launch_variant<T, 4, VP, false>(ix, a, sm_count, st);
}

template <typename T>
cudaError_t launch_typed(const DeviceIndex& ix, const SearchArgs& a, int sm_count, cudaStream_t st) {
  if (vp_for(ix.dim) == 4) return launch_vp<T, 4>(ix, a, sm_count, st);
  return launch_vp<T, 32>(ix, a, sm_count, st);
}

// ---------------------------------------------------------------------------
// Host-driven search, one hop per launch (the reference's SSD-hybrid mode:
// init_search + get_entry_kernel_inner, then per hop merge_data_kernel +
// unify_kernel; src/hyd_task_runner.cu:12-15,55-66,126-178,
// src/impl/hyd_search_v2.cuh:8-472). The caller supplies, per query, the 4 KB
// page holding the record of the node the previous step asked for. As in the
// reference's hybrid mode, the pivot-graph entry is searched with q'' (the
// query after init_query's in-place q -= c ... q += c), and so is the re-rank.
// Not a throughput path: the state of every query lives in device memory
// between launches, one warp works on one query.

// Query setup: q'' and the ADC table of each query, its entry node, empty
// pool and top-k.
template <typename T, bool IP>
__global__ void __launch_bounds__(128) hop_begin_kernel(const DeviceIndex ix, const float* __restrict__ q,
                                                        const HopState s) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp, wpb = blockDim.x / kWarp;
  const int dpad = (ix.dim + 3) & ~3;
  float* qc = reinterpret_cast<float*>(smem) + static_cast<size_t>(warp) * 2 * dpad;
  float* qs = qc + dpad;
  for (int64_t qid = static_cast<int64_t>(blockIdx.x) * wpb + warp; qid < s.nq;
       qid += static_cast<int64_t>(gridDim.x) * wpb) {
    const float* qq = q + qid * ix.dim;
    float* qpp = s.qpp + qid * ix.dim;
    for (int i = lane; i < ix.dim; i += kWarp) {
      const float c = __ldg(ix.centroid + i);
      const float d = IP ? qq[i] : __fsub_rn(qq[i], c);
      const float r = IP ? qq[i] : __fadd_rn(d, c);
      qc[i] = d;
      qs[i] = r;
      qpp[i] = r;
    }
    __syncwarp();
    build_lut<IP>(ix, qc, s.lut + qid * ix.chunks * kPivots, lane);
    uint32_t entry = static_cast<uint32_t>(ix.medoid);
    if (ix.has_nav) {
      bool capped = false;
      const int si = nav_search<T, IP>(ix, qs, lane, s.nav_max_hops, capped);
      const bool bad = si < 0 || si >= ix.nav_points;
      if (!bad) entry = static_cast<uint32_t>(__ldg(ix.nav_map + si));
      if ((capped || bad) && lane == 0) atomicAdd(s.err + 1, 1);
    }
    if (lane == 0) {
      s.request[qid] = static_cast<int32_t>(entry);
      s.psize[qid] = 0;
      s.found[qid] = 0;
      s.hops[qid] = 0;
    }
    for (int t = lane; t < s.topk; t += kWarp) {
      s.nns[qid * s.topk + t] = 0;
      s.dist[qid * s.topk + t] = 0.f;
    }
    __syncwarp();
  }
}

// One hop of every query that has a request: exact distance of the requested
// node u (re-rank), ADC of its neighbours, merge into the pool (first `ef`
// distinct entries of merge(pool, sorted neighbours), pool copy first), and
// the next request = the first unvisited pool entry (-1: the query is done).
// Neighbour ids past the index, or a degree past the slots, count as bad
// records (err[2]) and are dropped.
template <typename T, bool IP>
__global__ void __launch_bounds__(128) hop_step_kernel(const DeviceIndex ix, const HopState s,
                                                       const uint8_t* __restrict__ pages, int node_len, int npp) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp, wpb = blockDim.x / kWarp;
  const int R = ix.degree, L = s.ef, M = ix.chunks;
  uint64_t* nk = reinterpret_cast<uint64_t*>(smem) + static_cast<size_t>(warp) * (2 * R + L);
  uint64_t* mg = nk + R;
  for (int64_t qid = static_cast<int64_t>(blockIdx.x) * wpb + warp; qid < s.nq;
       qid += static_cast<int64_t>(gridDim.x) * wpb) {
    const int32_t u = s.request[qid];
    if (u < 0) continue;
    const uint32_t h = s.hops[qid] + 1;
    if (h > static_cast<uint32_t>(s.max_hops)) {
      if (lane == 0) {
        s.request[qid] = -1;
        atomicAdd(s.err, 1);
      }
      continue;
    }
    const uint8_t* rec = pages + qid * kPageSize + static_cast<size_t>(u % npp) * node_len;
    const T* vec = reinterpret_cast<const T*>(rec);
    const uint32_t* nbr = reinterpret_cast<const uint32_t*>(rec + static_cast<size_t>(ix.dim) * sizeof(T));
    int deg = static_cast<int>(nbr[0]);
    if (deg < 0 || deg > R) {
      if (lane == 0) atomicAdd(s.err + 2, 1);
      deg = deg < 0 ? 0 : R;
    }
    // re-rank u on q'' and insert after every equal top-k entry (retset_push_32):
    // the insertion point counted with ballots, the tail moved by all lanes
    const float ex = warp_dist<T, IP>(s.qpp + qid * ix.dim, vec, ix.dim, lane);
    {
      const int cnt = s.found[qid];
      int32_t* nn = s.nns + qid * s.topk;
      float* dd = s.dist + qid * s.topk;
      int le = 0;
      for (int t0 = 0; t0 < cnt; t0 += kWarp)
        le += __popc(__ballot_sync(kFull, t0 + lane < cnt && dd[t0 + lane] <= ex));
      if (le < s.topk) {
        const int hi = min(cnt, s.topk - 1);   // entries [le, hi) move one slot right
        for (int c = (hi - le + kWarp - 1) / kWarp - 1; c >= 0; --c) {
          const int t = le + c * kWarp + lane;
          float dv = 0.f;
          int iv = 0;
          if (t < hi) {
            dv = dd[t];
            iv = nn[t];
          }
          __syncwarp();
          if (t < hi) {
            dd[t + 1] = dv;
            nn[t + 1] = iv;
          }
          __syncwarp();
        }
        if (lane == 0) {
          dd[le] = ex;
          nn[le] = u;
        }
      }
      if (lane == 0) s.found[qid] = min(cnt + 1, s.topk);
    }
    // ADC of the neighbours, chunks in order; code rows read 16 bytes at a time
    const float* lut = s.lut + qid * M * kPivots;
    for (int e = lane; e < deg; e += kWarp) {
      const uint32_t v = nbr[1 + e];
      if (v >= static_cast<uint64_t>(ix.n)) {
        atomicAdd(s.err + 2, 1);
        nk[e] = ~0ull;
        continue;
      }
      const uint4* code = reinterpret_cast<const uint4*>(ix.codes + static_cast<size_t>(v) * ix.code_stride);
      float d = 0.f;
      for (int w = 0; w * 16 < M; ++w) d = adc16(d, __ldg(code + w), lut + 16 * w * kPivots, min(16, M - 16 * w));
      nk[e] = make_key(d, v);
    }
    __syncwarp();
    // a neighbour equal to a pool entry is dropped (the pool copy is kept)
    const int ps = s.psize[qid];
    uint64_t* pool = s.pool + qid * L;
    for (int e = lane; e < deg; e += kWarp) {
      if (nk[e] == ~0ull) continue;
      const uint64_t kk = nk[e] >> 1;
      int lo = 0, hi = ps;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((pool[mid] >> 1) < kk) lo = mid + 1; else hi = mid;
      }
      if (lo < ps && (pool[lo] >> 1) == kk) nk[e] = ~0ull;
    }
    __syncwarp();
    int nsv = 0;
    for (int e0 = 0; e0 < deg; e0 += kWarp) nsv += __popc(__ballot_sync(kFull, e0 + lane < deg && nk[e0 + lane] != ~0ull));
    // merged positions: pool entry i -> i + #survivors below it; survivor e ->
    // #survivors below it (ties by slot) + #pool entries below it
    for (int i = lane; i < ps; i += kWarp) {
      const uint64_t kk = pool[i] >> 1;
      int below = 0;
      for (int f = 0; f < deg; ++f) below += nk[f] != ~0ull && (nk[f] >> 1) < kk;
      if (i + below < L) mg[i + below] = pool[i];
    }
    for (int e = lane; e < deg; e += kWarp) {
      if (nk[e] == ~0ull) continue;
      const uint64_t kk = nk[e] >> 1;
      int below = 0;
      for (int f = 0; f < deg; ++f)
        below += nk[f] != ~0ull && ((nk[f] >> 1) < kk || ((nk[f] >> 1) == kk && f < e));
      int lo = 0, hi = ps;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((pool[mid] >> 1) < kk) lo = mid + 1; else hi = mid;
      }
      if (below + lo < L) mg[below + lo] = nk[e];
    }
    __syncwarp();
    const int nsz = min(ps + nsv, L);
    // next request: the first unvisited entry
    int first = -1;
    for (int j0 = 0; j0 < nsz; j0 += kWarp) {
      const unsigned bm = __ballot_sync(kFull, j0 + lane < nsz && (mg[j0 + lane] & 1ull));
      if (bm) {
        first = j0 + __ffs(bm) - 1;
        break;
      }
    }
    for (int j = lane; j < nsz; j += kWarp) pool[j] = j == first ? (mg[j] & ~1ull) : mg[j];
    if (lane == 0) {
      s.psize[qid] = nsz;
      s.hops[qid] = h;
      s.request[qid] = first >= 0 ? static_cast<int32_t>(static_cast<uint32_t>(mg[first]) >> 1) : -1;
    }
    __syncwarp();
  }
}

}  // namespace

cudaError_t launch_gather_neighbour_codes(const uint32_t* adj, int adj_stride, int degree, const uint8_t* codes,
                                          int code_stride, int64_t n, uint8_t* out, cudaStream_t st) {
  gather_neighbour_codes<<<148 * 8, 256, 0, st>>>(adj, adj_stride, degree, reinterpret_cast<const uint4*>(codes),
                                                  code_stride / 16, n, reinterpret_cast<uint4*>(out));
  return cudaGetLastError();
}

cudaError_t launch_hop_begin(const DeviceIndex& ix, const float* d_q, const HopState& s, int dtype,
                             cudaStream_t st) {
  if (s.nq <= 0) return cudaSuccess;
  const int wpb = 4;
  const size_t smem = sizeof(float) * 2 * ((ix.dim + 3) & ~3) * wpb;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((s.nq + wpb - 1) / wpb, 148 * 16));
  const bool ip = ix.metric == GANN_METRIC_IP;
  if (dtype == 0) {
    if (ip) hop_begin_kernel<uint8_t, true><<<grid, kWarp * wpb, smem, st>>>(ix, d_q, s);
    else hop_begin_kernel<uint8_t, false><<<grid, kWarp * wpb, smem, st>>>(ix, d_q, s);
  } else {
    if (ip) hop_begin_kernel<float, true><<<grid, kWarp * wpb, smem, st>>>(ix, d_q, s);
    else hop_begin_kernel<float, false><<<grid, kWarp * wpb, smem, st>>>(ix, d_q, s);
  }
  return cudaGetLastError();
}

cudaError_t launch_hop_step(const DeviceIndex& ix, const HopState& s, const uint8_t* d_pages, int32_t node_len,
                            int32_t nodes_per_page, int dtype, cudaStream_t st) {
  if (s.nq <= 0) return cudaSuccess;
  const int wpb = 4;
  const size_t smem = sizeof(uint64_t) * (2 * static_cast<size_t>(ix.degree) + s.ef) * wpb;
  const bool ip = ix.metric == GANN_METRIC_IP;
  auto fn = dtype == 0 ? (ip ? hop_step_kernel<uint8_t, true> : hop_step_kernel<uint8_t, false>)
                       : (ip ? hop_step_kernel<float, true> : hop_step_kernel<float, false>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((s.nq + wpb - 1) / wpb, 148 * 16));
  fn<<<grid, kWarp * wpb, smem, st>>>(ix, s, d_pages, node_len, nodes_per_page);
  return cudaGetLastError();
}

int search_max_ef() { return 32 * kWarp; }

int make_pivot_table(const std::vector<float>& pivots_t, const std::vector<int32_t>& chunk_off, int dim,
                     std::vector<float>& out) {
  const int m = static_cast<int>(chunk_off.size()) - 1;
  int maxw = 0;
  bool all3 = true;
  for (int c = 0; c < m; ++c) {
    const int w = chunk_off[c + 1] - chunk_off[c];
    maxw = std::max(maxw, w);
    all3 = all3 && w == 3;
  }
  if (m <= 0 || maxw > 4 || static_cast<int64_t>(pivots_t.size()) < static_cast<int64_t>(dim) * kPivots) return 0;
  out.assign(static_cast<size_t>(m) * kPivots * 4, 0.f);
  for (int c = 0; c < m; ++c)
    for (int j = 0; j < kPivots; ++j)
      for (int i = 0; i < chunk_off[c + 1] - chunk_off[c]; ++i)
        out[(static_cast<size_t>(c) * kPivots + j) * 4 + i] =
            pivots_t[static_cast<size_t>(chunk_off[c] + i) * kPivots + j];
  return all3 ? 3 : 4;
}

size_t search_smem_bytes(const DeviceIndex& ix, int topk, int ef) {
  return carve(nullptr, ix.chunks, ix.dim, npl_for(ix.degree), pl_for(ef), topk, nullptr);
}

cudaError_t launch_search(const DeviceIndex& ix, const SearchArgs& a, int dtype, int sm_count,
                          cudaStream_t st) {
  if (dtype == GANN_UINT8) return launch_typed<uint8_t>(ix, a, sm_count, st);
  return launch_typed<float>(ix, a, sm_count, st);
}

cudaError_t launch_probe_lut(const DeviceIndex& ix, const float* d_q, int64_t nq, float* d_lut,
                             cudaStream_t st) {
  const size_t smem = sizeof(float) * ((ix.dim + 3) & ~3);
  const unsigned grid = static_cast<unsigned>(nq < 65535 ? nq : 65535);
  if (grid == 0) return cudaSuccess;
  if (ix.metric == GANN_METRIC_IP) probe_lut_kernel<true><<<grid, kWarp, smem, st>>>(ix, d_q, nq, d_lut);
  else probe_lut_kernel<false><<<grid, kWarp, smem, st>>>(ix, d_q, nq, d_lut);
  return cudaGetLastError();
}

cudaError_t launch_probe_entry(const DeviceIndex& ix, const float* d_q, int64_t nq, int dtype,
                               int32_t* d_sample, int32_t* d_entry, int32_t* d_err, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((ix.dim + 3) & ~3);
  const unsigned grid = static_cast<unsigned>(nq < 65535 ? nq : 65535);
  if (grid == 0) return cudaSuccess;
  const int cap = 1 << 20;
  const bool ip = ix.metric == GANN_METRIC_IP;
  auto fn = dtype == GANN_UINT8 ? (ip ? probe_entry_kernel<uint8_t, true> : probe_entry_kernel<uint8_t, false>)
                                : (ip ? probe_entry_kernel<float, true> : probe_entry_kernel<float, false>);
  fn<<<grid, kWarp, smem, st>>>(ix, d_q, nq, d_sample, d_entry, d_err, cap);
  return cudaGetLastError();
}

}  // namespace gann
