// Index-file parsing for the search path. Same byte layouts as the reference
// loaders; every field is validated and a bad file yields GANN_EINVAL/GANN_EIO
// with a message instead of exit()/abort().
#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>

#include "gann_internal.hpp"

namespace gann {
namespace {

struct File {
  int fd = -1;
  int64_t size = 0;
  explicit File(const std::string& p) {
    fd = ::open(p.c_str(), O_RDONLY);
    if (fd >= 0) {
      struct stat st;
      if (fstat(fd, &st) == 0) size = st.st_size;
    }
  }
  ~File() {
    if (fd >= 0) ::close(fd);
  }
  bool ok() const { return fd >= 0; }
  bool read_at(void* dst, int64_t bytes, int64_t off) const {
    char* p = static_cast<char*>(dst);
    while (bytes > 0) {
      ssize_t r = ::pread(fd, p, static_cast<size_t>(std::min<int64_t>(bytes, 1 << 30)), off);
      if (r <= 0) {
        if (r < 0 && errno == EINTR) continue;
        return false;
      }
      p += r;
      off += r;
      bytes -= r;
    }
    return true;
  }
};

int fail(std::string& msg, int code, const std::string& m) {
  msg = m;
  return code;
}

// `bin` block: int32 npts, int32 ndim (src/pq_search.cu:187-201)
bool read_bin_head(const File& f, int64_t off, int32_t& npts, int32_t& ndim) {
  int32_t h[2];
  if (off < 0 || off + 8 > f.size || !f.read_at(h, 8, off)) return false;
  npts = h[0];
  ndim = h[1];
  return true;
}

}  // namespace

int load_disk_header(const std::string& path, int elem, HostIndex& hi, std::string& msg) {
  File f(path);
  if (!f.ok()) return fail(msg, GANN_EIO, "cannot open index file: " + path);
  // u32 nr, u32 nc, then u64 nnodes, ndims, medoid, max_node_len,
  // nnodes_per_sector, num_frozen, frozen_id, reorder_exists (src/layout.cpp:25-54)
  uint32_t head[2];
  uint64_t v[8];
  if (f.size < kPageSize || !f.read_at(head, 8, 0) || !f.read_at(v, sizeof(v), 8))
    return fail(msg, GANN_EIO, "index file shorter than its 4 KB header: " + path);
  const int64_t n = static_cast<int64_t>(v[0]), d = static_cast<int64_t>(v[1]);
  const int64_t node_len = static_cast<int64_t>(v[3]), npp = static_cast<int64_t>(v[4]);
  if (n <= 0 || n >= (int64_t(1) << 31))
    return fail(msg, GANN_EINVAL, "index header: node count out of range (1 .. 2^31-1)");
  if (d <= 0 || d > 4096) return fail(msg, GANN_EINVAL, "index header: bad dimension");
  const int64_t data_size = d * elem;
  if (node_len <= data_size + 4 || (node_len - data_size) % 4 != 0 || node_len > kPageSize)
    return fail(msg, GANN_EINVAL, "index header: record length inconsistent with dimension/type");
  if (npp <= 0 || npp * node_len > kPageSize)
    return fail(msg, GANN_EINVAL, "index header: nodes per page inconsistent with record length");
  if (static_cast<int64_t>(v[2]) < 0 || static_cast<int64_t>(v[2]) >= n)
    return fail(msg, GANN_EINVAL, "index header: medoid out of range");
  hi.elem = elem;
  hi.num_points = n;
  hi.dim = d;
  hi.medoid = static_cast<int64_t>(v[2]);
  hi.max_node_len = node_len;
  hi.nodes_per_page = npp;
  hi.data_size = data_size;
  hi.max_m0 = (node_len - data_size) / 4 - 1;   // src/layout.cpp:46
  hi.num_pages = (n + npp - 1) / npp;
  if (hi.max_m0 < 1 || hi.max_m0 > 128)
    return fail(msg, GANN_EUNSUPPORTED, "index: max degree must be in [1, 128]");
  if (f.size < (hi.num_pages + 1) * kPageSize)
    return fail(msg, GANN_EIO, "index file truncated: fewer pages than the header announces");
  return GANN_OK;
}

int load_pq(const std::string& prefix, HostIndex& hi, std::vector<uint8_t>& codes, int64_t& code_rows,
            std::string& msg) {
  const std::string piv = prefix + "_pivots.bin", cmp = prefix + "_compressed.bin";
  File fc(cmp);
  if (!fc.ok()) return fail(msg, GANN_EIO, "cannot open PQ codes: " + cmp);
  int32_t npts = 0, m = 0;
  if (!read_bin_head(fc, 0, npts, m)) return fail(msg, GANN_EIO, "PQ codes: short header");
  if (npts != hi.num_points) return fail(msg, GANN_EINVAL, "PQ codes: row count differs from the index");
  if (m <= 0 || m > 128) return fail(msg, GANN_EUNSUPPORTED, "PQ codes: chunk count must be in [1, 128]");
  if (fc.size < 8 + int64_t(npts) * m) return fail(msg, GANN_EIO, "PQ codes: file truncated");

  File fp(piv);
  if (!fp.ok()) return fail(msg, GANN_EIO, "cannot open PQ pivots: " + piv);
  int32_t nr = 0, nc = 0;
  if (!read_bin_head(fp, 0, nr, nc)) return fail(msg, GANN_EIO, "PQ pivots: short offsets table");
  if (!((nr == 4 || nr == 5) && nc == 1))
    return fail(msg, GANN_EINVAL, "PQ pivots: offsets table must be 4x1 or 5x1");   // src/pq_search.cu:80-83
  uint64_t offs[5];
  if (!fp.read_at(offs, 8 * nr, 8)) return fail(msg, GANN_EIO, "PQ pivots: short offsets table");
  int32_t pr = 0, pd = 0;
  if (!read_bin_head(fp, static_cast<int64_t>(offs[0]), pr, pd) || pr != kPivots || pd != hi.dim)
    return fail(msg, GANN_EINVAL, "PQ pivots: expected 256 x dim pivot table");
  std::vector<float> piv_rows(static_cast<size_t>(kPivots) * pd);
  if (!fp.read_at(piv_rows.data(), 4 * static_cast<int64_t>(piv_rows.size()), static_cast<int64_t>(offs[0]) + 8))
    return fail(msg, GANN_EIO, "PQ pivots: truncated pivot table");
  int32_t cr = 0, cc = 0;
  if (!read_bin_head(fp, static_cast<int64_t>(offs[1]), cr, cc) || cr != hi.dim || cc != 1)
    return fail(msg, GANN_EINVAL, "PQ pivots: expected dim x 1 centroid");
  hi.centroid.resize(hi.dim);
  if (!fp.read_at(hi.centroid.data(), 4 * hi.dim, static_cast<int64_t>(offs[1]) + 8))
    return fail(msg, GANN_EIO, "PQ pivots: truncated centroid");
  const int64_t co = static_cast<int64_t>(nr == 5 ? offs[3] : offs[2]);   // src/pq_search.cu:95-105
  int32_t orow = 0, ocol = 0;
  if (!read_bin_head(fp, co, orow, ocol) || orow != m + 1 || ocol != 1)
    return fail(msg, GANN_EINVAL, "PQ pivots: chunk offsets must be (M+1) x 1");
  std::vector<uint32_t> off(m + 1);
  if (!fp.read_at(off.data(), 4 * (m + 1), co + 8)) return fail(msg, GANN_EIO, "PQ pivots: truncated chunk offsets");
  // every dimension must belong to exactly one chunk: the reference indexes its
  // table with chunk_id = -1 otherwise (src/pq_search.cu:111-117)
  if (off[0] != 0 || off[m] != static_cast<uint32_t>(hi.dim))
    return fail(msg, GANN_EINVAL, "PQ pivots: chunk offsets must span [0, dim]");
  for (int i = 0; i < m; ++i)
    if (off[i + 1] <= off[i]) return fail(msg, GANN_EINVAL, "PQ pivots: chunk offsets must increase");
  hi.num_chunks = m;
  hi.chunk_offsets.assign(off.begin(), off.end());
  // transpose to [dim x 256] like PQSearch::read_data (src/pq_search.cu:88-93)
  hi.pivots_t.resize(static_cast<size_t>(hi.dim) * kPivots);
  for (int i = 0; i < kPivots; ++i)
    for (int64_t j = 0; j < hi.dim; ++j)
      hi.pivots_t[static_cast<size_t>(j) * kPivots + i] = piv_rows[static_cast<size_t>(i) * hi.dim + j];

  // codes, rows padded to 16 bytes
  const int64_t stride = round_up(m, 16);
  code_rows = npts;
  codes.assign(static_cast<size_t>(npts) * stride, 0);
  if (stride == m) {
    if (!fc.read_at(codes.data(), int64_t(npts) * m, 8)) return fail(msg, GANN_EIO, "PQ codes: read failed");
  } else {
    const int64_t blk = 1 << 20;
    std::vector<uint8_t> tmp(static_cast<size_t>(blk) * m);
    for (int64_t r0 = 0; r0 < npts; r0 += blk) {
      const int64_t rows = std::min<int64_t>(blk, npts - r0);
      if (!fc.read_at(tmp.data(), rows * m, 8 + r0 * m)) return fail(msg, GANN_EIO, "PQ codes: read failed");
      for (int64_t r = 0; r < rows; ++r)
        std::memcpy(&codes[static_cast<size_t>((r0 + r) * stride)], &tmp[static_cast<size_t>(r * m)], m);
    }
  }
  return GANN_OK;
}

int load_nav(const std::string& dir, HostIndex& hi, std::string& msg) {
  const std::string fdata = dir + "/nav_index.data", fmap = dir + "/map.txt", fidx = dir + "/nav_index";
  File fd(fdata);
  if (!fd.ok()) return fail(msg, GANN_EIO, "cannot open nav data: " + fdata);
  int32_t s = 0, d = 0;
  if (!read_bin_head(fd, 0, s, d)) return fail(msg, GANN_EIO, "nav data: short header");
  if (s <= 0) return fail(msg, GANN_EINVAL, "nav data: empty sample");
  if (d != hi.dim) return fail(msg, GANN_EINVAL, "nav data: dimension differs from the index");
  const int64_t row = d * hi.elem;
  if (fd.size < 8 + int64_t(s) * row) return fail(msg, GANN_EIO, "nav data: file truncated");
  const int64_t stride = round_up(d, 32) * hi.elem;
  hi.nav_vecs.assign(static_cast<size_t>(s) * stride, 0);
  {
    std::vector<uint8_t> tmp(static_cast<size_t>(s) * row);
    if (!fd.read_at(tmp.data(), int64_t(s) * row, 8)) return fail(msg, GANN_EIO, "nav data: read failed");
    for (int64_t i = 0; i < s; ++i)
      std::memcpy(&hi.nav_vecs[static_cast<size_t>(i * stride)], &tmp[static_cast<size_t>(i * row)], row);
  }
  // map.txt: sample index -> global id (src/nav_graph.cu:56-67)
  FILE* fm = std::fopen(fmap.c_str(), "r");
  if (!fm) return fail(msg, GANN_EIO, "cannot open nav map: " + fmap);
  hi.nav_map.resize(s);
  for (int32_t i = 0; i < s; ++i) {
    long long x = 0;
    if (std::fscanf(fm, "%lld", &x) != 1) {
      std::fclose(fm);
      return fail(msg, GANN_EINVAL, "nav map: fewer ids than samples");
    }
    if (x < 0 || x >= hi.num_points) {
      std::fclose(fm);
      return fail(msg, GANN_EINVAL, "nav map: id out of range of the index");
    }
    hi.nav_map[i] = static_cast<int32_t>(x);
  }
  std::fclose(fm);
  // nav_index: 24-byte header (max_m at byte 8, start at byte 12), then per node
  // u32 d, u32 nbr[d] (src/nav_graph.cu:68-95)
  File fi(fidx);
  if (!fi.ok()) return fail(msg, GANN_EIO, "cannot open nav graph: " + fidx);
  int32_t h[6];
  if (!fi.read_at(h, 24, 0)) return fail(msg, GANN_EIO, "nav graph: short header");
  const int32_t max_m = h[2], start = h[3];
  if (max_m <= 0 || max_m > kNavSlots) return fail(msg, GANN_EINVAL, "nav graph: max degree must be in [1, 32]");
  if (start < 0 || start >= s) return fail(msg, GANN_EINVAL, "nav graph: start node out of range");
  // rows of max_m slots, -1 padded, plus a tail of -1 so that a scan of 28
  // slots from the last row stays inside the array
  hi.nav_adj.assign(static_cast<size_t>(s) * max_m + kNavSlots, -1);
  std::vector<int32_t> words(static_cast<size_t>((fi.size - 24) / 4));
  if (!words.empty() && !fi.read_at(words.data(), 4 * int64_t(words.size()), 24))
    return fail(msg, GANN_EIO, "nav graph: read failed");
  size_t p = 0;
  for (int32_t i = 0; i < s; ++i) {
    if (p >= words.size()) return fail(msg, GANN_EIO, "nav graph: truncated");
    const int32_t k = words[p++];
    if (k <= 0 || k > max_m) return fail(msg, GANN_EINVAL, "nav graph: node degree out of range");
    if (p + k > words.size()) return fail(msg, GANN_EIO, "nav graph: truncated");
    for (int32_t j = 0; j < k; ++j) {
      const int32_t v = words[p + j];
      if (v < 0 || v >= s) return fail(msg, GANN_EINVAL, "nav graph: neighbour id out of range");
      hi.nav_adj[static_cast<size_t>(i) * max_m + j] = v;
    }
    p += k;
  }
  hi.has_nav = true;
  hi.nav_points = s;
  hi.nav_max_m = max_m;
  hi.nav_start = start;
  return GANN_OK;
}

int relayout_records(const std::string& path, const HostIndex& hi, int64_t first, int64_t count,
                     uint8_t* vec_out, int64_t vec_stride, uint32_t* adj_out, int32_t adj_stride,
                     std::string& msg) {
  if (count <= 0) return GANN_OK;
  File f(path);
  if (!f.ok()) return fail(msg, GANN_EIO, "cannot open index file: " + path);
  const int64_t npp = hi.nodes_per_page, nl = hi.max_node_len;
  const int64_t p0 = first / npp, p1 = (first + count - 1) / npp;
  std::vector<uint8_t> pages(static_cast<size_t>((p1 - p0 + 1) * kPageSize));
  // record i lives at 4096 * (1 + i / npp) + (i % npp) * node_len
  // (src/impl/pure_mem.cuh:261-265; page 0 is the header)
  if (!f.read_at(pages.data(), int64_t(pages.size()), (p0 + 1) * kPageSize))
    return fail(msg, GANN_EIO, "index file: short read of record pages");
  const int64_t ds = hi.data_size, m0 = hi.max_m0, n = hi.num_points;
  const unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  std::vector<int> bad(nt, 0);
  auto work = [&](unsigned t) {
    const int64_t a = count * t / nt, b = count * (t + 1) / nt;
    for (int64_t r = a; r < b; ++r) {
      const int64_t i = first + r;
      const uint8_t* rec = &pages[static_cast<size_t>((i / npp - p0) * kPageSize + (i % npp) * nl)];
      std::memcpy(vec_out + r * vec_stride, rec, ds);
      uint32_t deg;
      std::memcpy(&deg, rec + ds, 4);
      uint32_t* row = adj_out + r * adj_stride;
      if (deg > static_cast<uint32_t>(m0)) {
        bad[t] = 1;
        return;
      }
      std::memcpy(row, rec + ds + 4, 4 * static_cast<size_t>(deg));
      for (uint32_t j = 0; j < deg; ++j)
        if (row[j] >= static_cast<uint64_t>(n)) {
          bad[t] = 2;
          return;
        }
      for (int64_t j = deg; j < adj_stride; ++j) row[j] = kPadId;
    }
  };
  std::vector<std::thread> th;
  for (unsigned t = 1; t < nt; ++t) th.emplace_back(work, t);
  work(0);
  for (auto& x : th) x.join();
  for (int b : bad) {
    if (b == 1) return fail(msg, GANN_EINVAL, "index: a record's degree exceeds the neighbour slots");
    if (b == 2) return fail(msg, GANN_EINVAL, "index: a neighbour id is out of range");
  }
  return GANN_OK;
}

}  // namespace gann
