// check_recall -- recall@k of a search result file against a ground truth
// (the reference's bin/check_recall.cpp:11-32 tool, same arguments and output):
//
//   check_recall OUTPUT_BIN GROUND_TRUTH_IVECS
//
// OUTPUT_BIN is a `bin` file of int32 ids (int32 npts, int32 k, then npts x k
// ids; search_mem --output writes one), GROUND_TRUTH_IVECS an ivecs file of at
// least k ids per query for the same npts queries. Prints "Recall @ k: r" with
// the set-intersection recall of bin/utils.hpp:104-116 (a repeated result id
// counts each time). Errors exit with status 1 and a message instead of the
// reference's exit(-1).
#include <sys/stat.h>

#include <cstdint>
#include <cstdio>
#include <set>
#include <string>
#include <vector>

namespace {

bool fail(const std::string& m) {
  std::fprintf(stderr, "check_recall: %s\n", m.c_str());
  return false;
}

// ivecs: per row int32 d, then d int32 ids
bool read_ivecs(const char* path, std::vector<int32_t>& out, size_t& d, size_t& n) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(std::string("cannot open ") + path);
  struct stat st;
  fstat(fileno(f), &st);
  int32_t dd = 0;
  bool ok = std::fread(&dd, 4, 1, f) == 1 && dd > 0 && dd < 1000000;
  const size_t row = 4 + 4 * static_cast<size_t>(ok ? dd : 1);
  ok = ok && st.st_size % row == 0;
  if (ok) {
    d = static_cast<size_t>(dd);
    n = static_cast<size_t>(st.st_size) / row;
    std::vector<int32_t> raw(static_cast<size_t>(st.st_size) / 4);
    std::fseek(f, 0, SEEK_SET);
    ok = std::fread(raw.data(), 4, raw.size(), f) == raw.size();
    out.resize(n * d);
    for (size_t i = 0; ok && i < n; ++i) {
      if (raw[i * (d + 1)] != dd) ok = false;
      for (size_t j = 0; ok && j < d; ++j) out[i * d + j] = raw[i * (d + 1) + 1 + j];
    }
  }
  std::fclose(f);
  return ok ? true : fail(std::string(path) + ": not an ivecs file");
}

// bin: int32 npts, int32 ndims, then npts x ndims int32
bool read_bin(const char* path, std::vector<int32_t>& out, size_t& d, size_t& n) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(std::string("cannot open ") + path);
  struct stat st;
  fstat(fileno(f), &st);
  int32_t h[2] = {0, 0};
  bool ok = std::fread(h, 4, 2, f) == 2 && h[0] >= 0 && h[1] > 0 &&
            static_cast<int64_t>(st.st_size) == 8 + 4 * static_cast<int64_t>(h[0]) * h[1];
  if (ok) {
    n = static_cast<size_t>(h[0]);
    d = static_cast<size_t>(h[1]);
    out.resize(n * d);
    ok = std::fread(out.data(), 4, out.size(), f) == out.size();
  }
  std::fclose(f);
  return ok ? true : fail(std::string(path) + ": not a bin file of int32 ids");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    std::printf("%s: output_bin ground_truth_bin\n", argv[0]);
    return 1;
  }
  std::vector<int32_t> gt, res;
  size_t gd = 0, gn = 0, k = 0, rn = 0;
  if (!read_ivecs(argv[2], gt, gd, gn) || !read_bin(argv[1], res, k, rn)) return 1;
  if (gd < k) {
    std::printf("DIM mismatch: %zu vs %zu\n", gd, k);
    return 1;
  }
  if (gn != rn) {
    std::printf("NUM mismatch: %zu vs %zu\n", gn, rn);
    return 1;
  }
  size_t cnt = 0;
  for (size_t i = 0; i < gn; ++i) {
    std::set<int32_t> s(gt.begin() + i * gd, gt.begin() + i * gd + k);
    for (size_t j = 0; j < k; ++j) cnt += s.count(res[i * k + j]);
  }
  std::printf("Recall @ %zu: %f\n", k, gn ? static_cast<double>(cnt) / (gn * k) : 0.0);
  return 0;
}
