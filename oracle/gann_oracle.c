/*
 * gann_oracle.c -- TEST INFRASTRUCTURE, not product code.
 *
 * A CPU restatement of the reference's in-memory search path (GustANN) used
 * only as the checker for the CUDA path (tests/, __graft_entry__.smoke(),
 * bench.py's CPU-baseline leg). Nothing in gustann_b200/ links or calls it.
 *
 * It parses the index files itself and replays the reference's steps
 * literally, one query per thread (OpenMP over queries):
 *   oracle_lut     PQSearchData::init_query          src/impl/pq.cuh:8-59
 *   warp_sq        square_sum_32                     src/impl/util.cuh:26-46
 *   oracle_nav     get_entry_kernel_inner + translate src/impl/nav.cuh:13-135,
 *                                                     src/nav_graph.cu:104-109
 *   search_one     search_graph_kernel_gpumem<T>     src/impl/pure_mem.cuh:243-432
 *                  lower_bound                       src/impl/util.cuh:166-178
 *                  retset_push_32                    src/impl/util.cuh:116-163
 * Loaders follow src/layout.cpp:11-69, src/pq_search.cu:56-121,187-201 and
 * src/nav_graph.cu:41-100.
 *
 * oracle_set_metric(o, 1) switches every distance to the inner product,
 * searched as -<q, x> (the reference is L2-only, src/common.hpp:28-30; this
 * is the definition the CUDA path follows): ADC entries -(sum of q_i * p_ji)
 * per chunk, exact distances -(lane-strided q.x sums, shfl tree), q'' = q.
 *
 * `fma_mode` selects how the reference's `acc += d * d` statements are
 * evaluated: 1 = fused multiply-add (nvcc's default contraction), 0 = separate
 * multiply and add. Compile with -ffp-contract=off so the C compiler adds no
 * contraction of its own.
 *
 * Per-query flags report inputs on which the reference's behaviour is not
 * defined: ORACLE_F_HOPCAP (hop cap reached), ORACLE_F_STALE (the reference
 * would read a stale pool slot), ORACLE_F_DUPNBR (repeated neighbour id), and
 * ORACLE_F_NAVRACE (two racing stores in the nav dedup with different values).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NPIV 256
#define ORACLE_F_HOPCAP 1
#define ORACLE_F_STALE 2
#define ORACLE_F_DUPNBR 4
#define ORACLE_F_NAVRACE 8
#define NAV_L 4
#define NAV_R 28

typedef struct {
  int dtype, elem, fma_mode;
  int metric; /* 0: squared L2 (the reference's), 1: inner product as -<q, x> */
  /* disk index */
  int64_t n, dim, medoid, node_len, npp, max_m0, data_size, num_pages;
  uint8_t* pages; /* num_pages * 4096, header page dropped */
  /* PQ */
  int m;
  float* pivots_t; /* [dim x 256] */
  float* centroid;
  int* chunk_id; /* [dim] */
  uint8_t* codes; /* [n x m] */
  /* nav */
  int has_nav;
  int64_t s;
  int nav_max_m, nav_start;
  uint8_t* nav_data; /* [s x dim] elements */
  int* nav_graph;    /* [s x max_m] + NAV_R tail of -1 */
  int* nav_map;
} oracle_t;

static float sqacc(float acc, float d, int fma_mode) {
  if (fma_mode) return fmaf(d, d, acc);
  {
    volatile float p = d * d;
    return acc + p;
  }
}

/* acc + a * b, fused or not like sqacc */
static float dotacc(float acc, float a, float b, int fma_mode) {
  if (fma_mode) return fmaf(a, b, acc);
  {
    volatile float p = a * b;
    return acc + p;
  }
}

static float elem_at(const oracle_t* o, const uint8_t* base, int64_t i) {
  if (o->dtype == 0) return (float)base[i];
  {
    float f;
    memcpy(&f, base + 4 * i, 4);
    return f;
  }
}

/* square_sum_32: lane l sums dims l, l+32, ...; then the shfl_down tree as
 * seen by lane 0 (src/impl/util.cuh:26-46). */
static float warp_sq(const oracle_t* o, const float* a, const uint8_t* b) {
  float p[32];
  int l, off;
  for (l = 0; l < 32; ++l) {
    float v = 0.f;
    int64_t i;
    for (i = l; i < o->dim; i += 32) {
      if (o->metric) {
        v = dotacc(v, a[i], elem_at(o, b, i), o->fma_mode);
      } else {
        float d = a[i] - elem_at(o, b, i);
        v = sqacc(v, d, o->fma_mode);
      }
    }
    p[l] = v;
  }
  for (off = 16; off > 0; off >>= 1)
    for (l = 0; l < off; ++l) p[l] = p[l] + p[l + off];
  /* inner product: the same lane sums and tree on q.x, negated */
  return o->metric ? -p[0] : p[0];
}

/* ------------------------------------------------------------- loading */

static int read_at(FILE* f, void* dst, size_t bytes, int64_t off) {
  if (fseek(f, (long)off, SEEK_SET) != 0) return -1;
  return fread(dst, 1, bytes, f) == bytes ? 0 : -1;
}

static int load_bin_head(FILE* f, int64_t off, int32_t* npts, int32_t* ndim) {
  int32_t h[2];
  if (read_at(f, h, 8, off)) return -1;
  *npts = h[0];
  *ndim = h[1];
  return 0;
}

void oracle_close(oracle_t* o) {
  if (!o) return;
  free(o->pages);
  free(o->pivots_t);
  free(o->centroid);
  free(o->chunk_id);
  free(o->codes);
  free(o->nav_data);
  free(o->nav_graph);
  free(o->nav_map);
  free(o);
}

oracle_t* oracle_open(const char* index_file, const char* pq_prefix, const char* nav_dir, int dtype,
                      int fma_mode) {
  oracle_t* o = (oracle_t*)calloc(1, sizeof(oracle_t));
  char path[4096];
  FILE* f;
  uint32_t head[2];
  uint64_t v[8];
  int32_t a, b;
  uint64_t offs[5];
  float* piv;
  uint32_t* co;
  int i, j;
  if (!o) return NULL;
  o->dtype = dtype;
  o->elem = dtype == 0 ? 1 : 4;
  o->fma_mode = fma_mode;
  /* disk index header (src/layout.cpp:25-54) */
  f = fopen(index_file, "rb");
  if (!f) goto fail;
  if (read_at(f, head, 8, 0) || read_at(f, v, sizeof(v), 8)) goto fail_f;
  o->n = (int64_t)v[0];
  o->dim = (int64_t)v[1];
  o->medoid = (int64_t)v[2];
  o->node_len = (int64_t)v[3];
  o->npp = (int64_t)v[4];
  o->data_size = o->dim * o->elem;
  o->max_m0 = (o->node_len - o->data_size) / 4 - 1;
  o->num_pages = (o->n + o->npp - 1) / o->npp;
  o->pages = (uint8_t*)malloc((size_t)o->num_pages * 4096);
  if (!o->pages || read_at(f, o->pages, (size_t)o->num_pages * 4096, 4096)) goto fail_f;
  fclose(f);

  /* PQ codes + pivots (src/pq_search.cu:56-121) */
  snprintf(path, sizeof(path), "%s_compressed.bin", pq_prefix);
  f = fopen(path, "rb");
  if (!f || load_bin_head(f, 0, &a, &b)) goto fail_f;
  o->m = b;
  o->codes = (uint8_t*)malloc((size_t)a * b);
  if (!o->codes || read_at(f, o->codes, (size_t)a * b, 8)) goto fail_f;
  fclose(f);
  snprintf(path, sizeof(path), "%s_pivots.bin", pq_prefix);
  f = fopen(path, "rb");
  if (!f || load_bin_head(f, 0, &a, &b) || !(a == 4 || a == 5) || read_at(f, offs, 8 * (size_t)a, 8)) goto fail_f;
  {
    int nr = a;
    int32_t pr, pd;
    if (load_bin_head(f, (int64_t)offs[0], &pr, &pd) || pr != NPIV || pd != o->dim) goto fail_f;
    piv = (float*)malloc(sizeof(float) * NPIV * o->dim);
    o->pivots_t = (float*)malloc(sizeof(float) * NPIV * o->dim);
    if (!piv || !o->pivots_t || read_at(f, piv, sizeof(float) * NPIV * o->dim, (int64_t)offs[0] + 8)) goto fail_f;
    for (i = 0; i < NPIV; ++i)
      for (j = 0; j < o->dim; ++j) o->pivots_t[(size_t)j * NPIV + i] = piv[(size_t)i * o->dim + j];
    free(piv);
    o->centroid = (float*)malloc(sizeof(float) * o->dim);
    if (read_at(f, o->centroid, sizeof(float) * o->dim, (int64_t)offs[1] + 8)) goto fail_f;
    co = (uint32_t*)malloc(sizeof(uint32_t) * (o->m + 1));
    if (read_at(f, co, sizeof(uint32_t) * (o->m + 1), (int64_t)(nr == 5 ? offs[3] : offs[2]) + 8)) goto fail_f;
    o->chunk_id = (int*)malloc(sizeof(int) * o->dim);
    for (j = 0; j < o->dim; ++j) o->chunk_id[j] = -1;
    for (i = 0; i < o->m; ++i)
      for (j = (int)co[i]; j < (int)co[i + 1]; ++j) o->chunk_id[j] = i;
    free(co);
  }
  fclose(f);

  /* nav graph (src/nav_graph.cu:41-100) */
  if (nav_dir && nav_dir[0]) {
    int32_t hh[6];
    int s;
    snprintf(path, sizeof(path), "%s/nav_index.data", nav_dir);
    f = fopen(path, "rb");
    if (!f || load_bin_head(f, 0, &a, &b)) goto fail_f;
    o->s = a;
    o->nav_data = (uint8_t*)malloc((size_t)a * b * o->elem);
    if (read_at(f, o->nav_data, (size_t)a * b * o->elem, 8)) goto fail_f;
    fclose(f);
    snprintf(path, sizeof(path), "%s/map.txt", nav_dir);
    f = fopen(path, "r");
    if (!f) goto fail;
    o->nav_map = (int*)malloc(sizeof(int) * o->s);
    for (s = 0; s < o->s; ++s)
      if (fscanf(f, "%d", &o->nav_map[s]) != 1) goto fail_f;
    fclose(f);
    snprintf(path, sizeof(path), "%s/nav_index", nav_dir);
    f = fopen(path, "rb");
    if (!f || read_at(f, hh, 24, 0)) goto fail_f;
    o->nav_max_m = hh[2];
    o->nav_start = hh[3];
    o->nav_graph = (int*)malloc(sizeof(int) * ((size_t)o->s * o->nav_max_m + NAV_R));
    for (i = 0; i < o->s * o->nav_max_m + NAV_R; ++i) o->nav_graph[i] = -1;
    for (s = 0; s < o->s; ++s) {
      int d;
      if (fread(&d, 4, 1, f) != 1 || d < 0 || d > o->nav_max_m) goto fail_f;
      if ((int)fread(o->nav_graph + (size_t)o->nav_max_m * s, 4, d, f) != d) goto fail_f;
    }
    fclose(f);
    o->has_nav = 1;
  }
  return o;
fail_f:
  if (f) fclose(f);
fail:
  oracle_close(o);
  return NULL;
}

/* PQSearchData::init_query: table lut[M x 256] and the restored query
 * q'' = (q - c) + c (src/impl/pq.cuh:8-59). */
static void lut_one(const oracle_t* o, const float* q, float* lut, float* qc, float* qpp) {
  int64_t i;
  int j;
  memset(lut, 0, sizeof(float) * o->m * NPIV);
  if (o->metric) {
    /* inner product (no counterpart in the reference): entry (c, j) =
     * -(sum over the chunk's dims, ascending, of q_i * pivot_ji), accumulated
     * from 0 like the L2 entries; the query is used as given (q'' = q) */
    for (i = 0; i < o->dim; ++i) {
      int idx = o->chunk_id[i];
      for (j = 0; j < NPIV; ++j)
        lut[idx * NPIV + j] = dotacc(lut[idx * NPIV + j], q[i], o->pivots_t[(size_t)i * NPIV + j], o->fma_mode);
    }
    for (j = 0; j < o->m * NPIV; ++j) lut[j] = -lut[j];
    for (i = 0; i < o->dim; ++i) {
      qc[i] = q[i];
      qpp[i] = q[i];
    }
    return;
  }
  for (i = 0; i < o->dim; ++i) qc[i] = q[i] - o->centroid[i];
  for (i = 0; i < o->dim; ++i) {
    int idx = o->chunk_id[i];
    for (j = 0; j < NPIV; ++j) {
      float d = qc[i] - o->pivots_t[(size_t)i * NPIV + j];
      lut[idx * NPIV + j] = sqacc(lut[idx * NPIV + j], d, o->fma_mode);
    }
  }
  for (i = 0; i < o->dim; ++i) qpp[i] = qc[i] + o->centroid[i];
}

void oracle_lut(const oracle_t* o, const float* q, int64_t nq, float* luts) {
  int64_t k;
#pragma omp parallel for schedule(static)
  for (k = 0; k < nq; ++k) {
    float* qc = (float*)malloc(sizeof(float) * o->dim * 2);
    lut_one(o, q + k * o->dim, luts + (size_t)k * o->m * NPIV, qc, qc + o->dim);
    free(qc);
  }
}

/* get_entry_kernel_inner (src/impl/nav.cuh:13-135), one warp emulated with
 * arrays of 32 slots. Returns the sample index; *flags gets ORACLE_F_NAVRACE
 * when racing stores with different values decide the result. */
static int nav_one(const oracle_t* o, const float* q, int max_hops, int* flags) {
  uint32_t id[32];
  float dist[32];
  int t, i, hop, idx = 0;
  const int64_t rowb = o->dim * o->elem;
  id[0] = (uint32_t)o->nav_start;
  dist[0] = warp_sq(o, q, o->nav_data + (size_t)o->nav_start * rowb);
  for (t = 1; t < 32; ++t) {
    id[t] = 0xffffffffu;
    dist[t] = INFINITY;
  }
  for (hop = 0; idx != -1; ++hop) {
    uint32_t u;
    const int* edge;
    unsigned val;
    int x;
    if (hop >= max_hops) {
      *flags |= ORACLE_F_HOPCAP;
      break;
    }
    u = id[idx];
    id[idx] |= 0x80000000u;
    edge = o->nav_graph + (size_t)o->nav_max_m * u;
    for (i = 0; i < NAV_R; ++i) {
      int v = edge[i];
      if (v == -1) break;
      id[i + NAV_L] = (uint32_t)v;
      dist[i + NAV_L] = warp_sq(o, q, o->nav_data + (size_t)v * rowb);
    }
    for (i = 0; i < NAV_L; ++i) {
      float ld[32];
      int pos[32], off, p, hi = -1, kill[32];
      uint32_t prev = i > 0 ? id[i - 1] : 0;
      for (t = 0; t < 32; ++t) {
        ld[t] = dist[t];
        pos[t] = t;
        kill[t] = 0;
        if (t < i) ld[t] = INFINITY;
        else if (i != 0 && ((id[t] ^ prev) & 0x7fffffffu) == 0) kill[t] = 1;
      }
      for (t = 0; t < 32; ++t)
        if (kill[t]) {
          if (hi >= 0 && ((id[hi] | prev) != (id[t] | prev))) *flags |= ORACLE_F_NAVRACE;
          hi = t;
        }
      /* every matching lane stores id[i-1] | id[tid]; the highest lane's store is taken */
      if (hi >= 0) id[i - 1] = prev | id[hi];
      for (t = 0; t < 32; ++t)
        if (kill[t]) ld[t] = dist[t] = INFINITY;
      /* shfl_down argmin tree: lane l takes lane l+off's pair if strictly smaller */
      for (off = 16; off > 0; off >>= 1)
        for (t = 0; t + off < 32; ++t)
          if (ld[t + off] < ld[t]) {
            ld[t] = ld[t + off];
            pos[t] = pos[t + off];
          }
      p = pos[0];
      if (i != p) {
        float tv = dist[i], yv = dist[p];
        if (tv != yv) {
          uint32_t m = id[i];
          dist[i] = yv;
          dist[p] = tv;
          id[i] = id[p];
          id[p] = m;
        }
      }
    }
    val = 0;
    for (t = 0; t < 32; ++t)
      if (!(id[t] & 0x80000000u)) val |= 1u << t;
    x = val ? __builtin_ctz(val) : 32;
    idx = x < NAV_L ? x : -1;
  }
  return (int)(id[0] & 0x7fffffffu);
}

void oracle_nav(const oracle_t* o, const float* q, int64_t nq, int32_t* sample, int32_t* entry, int32_t* flags) {
  int64_t k;
#pragma omp parallel for schedule(dynamic, 16)
  for (k = 0; k < nq; ++k) {
    int fl = 0;
    int s = nav_one(o, q + k * o->dim, 1 << 20, &fl);
    sample[k] = s;
    entry[k] = o->nav_map[s];
    if (flags) flags[k] = fl;
  }
}

/* lower_bound on (dist, id & 0x7fffffff) over [l, r) (src/impl/util.cuh:166-178) */
static int lower_bound(const float* d, const uint32_t* id, int l, int r, float x, uint32_t xi) {
  xi &= 0x7fffffffu;
  while (l < r) {
    int mid = (l + r) / 2;
    if (d[mid] < x || (d[mid] == x && (id[mid] & 0x7fffffffu) < xi)) l = mid + 1;
    else r = mid;
  }
  return l;
}

/* retset_push_32 as a sequential insert: the new value goes after every entry
 * that is <= it; the list keeps at most `topk` entries (src/impl/util.cuh:116-163). */
static void retset_push(float* dist, int* idx, int* size, int topk, float value, int vid) {
  int p = *size - 1;
  while (p >= 0 && dist[p] > value) {
    if (p + 1 < topk) {
      dist[p + 1] = dist[p];
      idx[p + 1] = idx[p];
    }
    --p;
  }
  if (p + 1 < topk) {
    dist[p + 1] = value;
    idx[p + 1] = vid;
  }
  if (*size + 1 <= topk) ++*size;
}

typedef struct {
  float* lut;
  float* qc;
  float* qpp;
  uint32_t* tmp_id;
  float* tmp_dist;
  uint32_t* mv_id;
  float* mv_dist;
  int* mv_pos;
  int* order;
} work_t;

static int cmp_key(const float* d, const uint32_t* id, int a, int b) {
  if (d[a] < d[b]) return -1;
  if (d[a] > d[b]) return 1;
  {
    uint32_t x = id[a] & 0x7fffffffu, y = id[b] & 0x7fffffffu;
    return x < y ? -1 : (x > y ? 1 : 0);
  }
}

/* search_graph_kernel_gpumem<T> for one query (src/impl/pure_mem.cuh:277-428). */
static void search_one(const oracle_t* o, const float* q, int64_t entry, int topk, int L, int max_hops,
                       int32_t* nns, float* dists, int32_t* found, uint32_t* hops_out, int* flags, work_t* w) {
  const int max_m = (int)o->max_m0;
  const int bdim = ((max_m + 31) / 32 * 32) > 64 ? ((max_m + 31) / 32 * 32) : 64;
  int ctx_size = 0, size = 0, hops = 0, i, t;
  int64_t u = entry;
  lut_one(o, q, w->lut, w->qc, w->qpp);
  for (t = 0; t < topk; ++t) {
    nns[t] = 0;
    dists[t] = 0.f;
  }
  while (u != -1) {
    const uint8_t* node;
    const uint32_t* meta;
    int deg, sz = ctx_size, s, count, id;
    float ex;
    if (hops >= max_hops) {
      *flags |= ORACLE_F_HOPCAP;
      break;
    }
    ++hops;
    node = o->pages + (size_t)(u / o->npp) * 4096 + (size_t)(u % o->npp) * o->node_len;
    meta = (const uint32_t*)(node + o->data_size);
    deg = (int)meta[0];
    for (t = 0; t < bdim; ++t) {
      if (t >= deg) {
        if (t < max_m) {
          w->tmp_id[sz + t] = 0xffffffffu - (uint32_t)t;
          w->tmp_dist[sz + t] = INFINITY;
        }
      } else {
        uint32_t v = meta[1 + t];
        const uint8_t* c = o->codes + (size_t)v * o->m;
        float dd = 0.f;
        int j;
        for (j = 0; j < o->m; ++j) dd += w->lut[j * NPIV + c[j]];
        w->tmp_id[sz + t] = v;
        w->tmp_dist[sz + t] = dd;
      }
    }
    /* merge-path rounds of src/impl/pure_mem.cuh:314-348 sort [sz, sz+deg) by
     * (dist, id); with distinct keys that is a plain sort */
    for (t = 0; t < deg; ++t) w->order[t] = t;
    for (t = 1; t < deg; ++t) { /* insertion sort on indices, stable */
      int k = w->order[t], r = t - 1;
      while (r >= 0 && cmp_key(w->tmp_dist + sz, w->tmp_id + sz, w->order[r], k) > 0) {
        w->order[r + 1] = w->order[r];
        --r;
      }
      w->order[r + 1] = k;
    }
    for (t = 1; t < deg; ++t)
      if (cmp_key(w->tmp_dist + sz, w->tmp_id + sz, w->order[t - 1], w->order[t]) == 0) *flags |= ORACLE_F_DUPNBR;
    for (t = 0; t < deg; ++t) {
      w->mv_id[t] = w->tmp_id[sz + w->order[t]];
      w->mv_dist[t] = w->tmp_dist[sz + w->order[t]];
    }
    for (t = 0; t < deg; ++t) {
      w->tmp_id[sz + t] = w->mv_id[t];
      w->tmp_dist[sz + t] = w->mv_dist[t];
    }
    /* external merge (src/impl/pure_mem.cuh:350-378) */
    for (t = 0; t < deg; ++t) {
      id = lower_bound(w->tmp_dist, w->tmp_id, 0, sz, w->tmp_dist[sz + t], w->tmp_id[sz + t]);
      if (id != sz && ((w->tmp_id[id] ^ w->tmp_id[sz + t]) & 0x7fffffffu) == 0) id++;
      w->mv_pos[sz + t] = id + t;
    }
    for (i = 0; i < sz; ++i) {
      id = lower_bound(w->tmp_dist + sz, w->tmp_id + sz, 0, deg, w->tmp_dist[i], w->tmp_id[i]);
      w->mv_pos[i] = id + i;
    }
    for (i = 0; i < sz + deg; ++i) {
      w->mv_id[w->mv_pos[i]] = w->tmp_id[i];
      w->mv_dist[w->mv_pos[i]] = w->tmp_dist[i];
    }
    ctx_size = sz + deg < 2 * L ? sz + deg : 2 * L;
    /* warp 0: dedup adjacent equal ids, first unvisited (src/impl/pure_mem.cuh:380-419) */
    s = ctx_size;
    id = s + 1;
    count = 0;
    for (i = 0; i < s; ++i) {
      int flag = (i != 0) && (((w->mv_id[i] ^ w->mv_id[i - 1]) & 0x7fffffffu) == 0);
      if (flag) {
        ++count;
        continue;
      }
      {
        int mvp = i - count;
        w->tmp_id[mvp] = w->mv_id[i];
        w->tmp_dist[mvp] = w->mv_dist[i];
        if (id > mvp && !(w->mv_id[i] & 0x80000000u)) id = mvp;
      }
    }
    /* warp 1: exact distance of u on q'' and top-k insert */
    ex = warp_sq(o, w->qpp, node);
    retset_push(dists, nns, &size, topk, ex, (int)u);
    if (id >= L) {
      u = -1;
    } else if (id >= s - count) {
      /* the reference would expand tmp_id[id], a slot this step did not write */
      *flags |= ORACLE_F_STALE;
      u = -1;
    } else {
      u = w->tmp_id[id];
      ctx_size = s - count < L ? s - count : L;
      w->tmp_id[id] |= 0x80000000u;
    }
  }
  *found = size;
  if (hops_out) *hops_out = (uint32_t)hops;
}

/* Full search of nq queries; `entries` (nullable) overrides the nav result. */
int oracle_search(const oracle_t* o, const float* q, int64_t nq, int topk, int L, int max_hops, const int32_t* entries,
                  int32_t* nns, float* dists, int32_t* found, uint32_t* hops, int32_t* flags, int nthreads) {
  int64_t k;
  int bad = 0;
  const int cap = L + (int)o->max_m0 + 64;
  const int nt = nthreads > 0 ? nthreads : omp_get_max_threads();
#pragma omp parallel num_threads(nt)
  {
    work_t w;
    w.lut = (float*)malloc(sizeof(float) * o->m * NPIV);
    w.qc = (float*)malloc(sizeof(float) * o->dim);
    w.qpp = (float*)malloc(sizeof(float) * o->dim);
    w.tmp_id = (uint32_t*)malloc(sizeof(uint32_t) * cap);
    w.tmp_dist = (float*)malloc(sizeof(float) * cap);
    w.mv_id = (uint32_t*)malloc(sizeof(uint32_t) * cap);
    w.mv_dist = (float*)malloc(sizeof(float) * cap);
    w.mv_pos = (int*)malloc(sizeof(int) * cap);
    w.order = (int*)malloc(sizeof(int) * cap);
#pragma omp for schedule(dynamic, 4)
    for (k = 0; k < nq; ++k) {
      int fl = 0;
      int64_t e;
      const float* qk = q + k * o->dim;
      if (entries) e = entries[k];
      else if (o->has_nav) e = o->nav_map[nav_one(o, qk, 1 << 20, &fl)];
      else e = o->medoid;
      search_one(o, qk, e, topk, L, max_hops, nns + k * topk, dists + k * topk, found + k,
                 hops ? hops + k : NULL, &fl, &w);
      if (flags) flags[k] = fl;
      if (fl) {
#pragma omp atomic
        bad++;
      }
    }
    free(w.lut);
    free(w.qc);
    free(w.qpp);
    free(w.tmp_id);
    free(w.tmp_dist);
    free(w.mv_id);
    free(w.mv_dist);
    free(w.mv_pos);
    free(w.order);
  }
  return bad;
}

int64_t oracle_dim(const oracle_t* o) { return o->dim; }
void oracle_set_metric(oracle_t* o, int metric) { o->metric = metric ? 1 : 0; }
int oracle_chunks(const oracle_t* o) { return o->m; }
