// search_mem -- command-line driver with the reference driver's flags and
// output table (bin/search_disk.cpp:51-73, 152-256; recall bin/utils.hpp:104-116),
// linked against libgann.so through the C++ facade.
//
//   search_mem --query Q --index I --pq_data P [--nav_graph N] --data_type uint8|float
//              [--ground_truth GT] [--topk K] --ef_search L [L2 ...] [-R repeat] [-G]
//              [--output FILE]
// --output writes the ids of the (last) ef_search as a `bin` file of int32
// (npts, k, ids), the result file check_recall reads.
#include <sys/stat.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "gustann.hpp"

namespace {

// vecs files: per row int32 d, then d elements of `elem` bytes
std::vector<uint8_t> read_vecs(const std::string& path, size_t elem, size_t& d, size_t& n) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    std::fprintf(stderr, "could not open %s\n", path.c_str());
    std::exit(1);
  }
  int32_t dd = 0;
  if (std::fread(&dd, 4, 1, f) != 1 || dd <= 0 || dd >= 1000000) {
    std::fprintf(stderr, "%s: unreasonable dimension\n", path.c_str());
    std::exit(1);
  }
  struct stat st;
  fstat(fileno(f), &st);
  const size_t row = 4 + static_cast<size_t>(dd) * elem;
  if (st.st_size % row) {
    std::fprintf(stderr, "%s: weird file size\n", path.c_str());
    std::exit(1);
  }
  d = dd;
  n = st.st_size / row;
  std::vector<uint8_t> raw(st.st_size), out(n * d * elem);
  std::fseek(f, 0, SEEK_SET);
  if (std::fread(raw.data(), 1, raw.size(), f) != raw.size()) {
    std::fprintf(stderr, "%s: short read\n", path.c_str());
    std::exit(1);
  }
  std::fclose(f);
  for (size_t i = 0; i < n; ++i) std::memcpy(&out[i * d * elem], &raw[i * row + 4], d * elem);
  return out;
}

// set-intersection recall@k (bin/utils.hpp:104-116)
double calc_recall(const int* res, const int* gt, size_t num, size_t dim, int k) {
  size_t cnt = 0;
  for (size_t i = 0; i < num; ++i) {
    std::set<int> s(gt + i * dim, gt + i * dim + k);
    for (int j = 0; j < k; ++j) cnt += s.count(res[i * k + j]);
  }
  return static_cast<double>(cnt) / (num * k);
}

void usage() {
  std::fprintf(stderr,
               "usage: search_mem --query FILE --index FILE --pq_data PREFIX --data_type uint8|float\n"
               "                  [--nav_graph DIR] [--ground_truth FILE] [--topk K]\n"
               "                  --ef_search L [L ...] [-R|--repeat N] [-G|--use-gpu-mem] [--device D]\n"
               "                  [--hybrid -B|--minibatch N -T|--thread N [--io_backend memory]]\n"
               "                  [--output FILE]  ids of the last ef_search as a bin file (check_recall)\n"
               "  --hybrid: records stay in the index file and each hop reads the needed pages\n"
               "            (the reference driver's HYBRID_CALC build, GustANN::init_hybrid)\n");
  std::exit(1);
}

}  // namespace

int main(int argc, char** argv) {
  std::string query_file, gt_file, data_type, out_file;
  gustann::GustANNConfig cfg;
  int topk = 100, repeat = 20, device = 0;
  bool use_gpu_mem = false, hybrid = false;
  gustann::HybridExecutorConfig hcfg;
  std::vector<int> efs;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto need = [&]() -> std::string {
      if (i + 1 >= argc) usage();
      return argv[++i];
    };
    if (a == "--query") query_file = need();
    else if (a == "--index") cfg.index_file = need();
    else if (a == "--ground_truth") gt_file = need();
    else if (a == "--data_type") data_type = need();
    else if (a == "--topk") topk = std::atoi(need().c_str());
    else if (a == "--pq_data") cfg.pq_file_prefix = need();
    else if (a == "--nav_graph") cfg.nav_graph_prefix = need();
    else if (a == "--repeat" || a == "-R") repeat = std::atoi(need().c_str());
    else if (a == "--use-gpu-mem" || a == "-G") use_gpu_mem = true;
    else if (a == "--device") device = std::atoi(need().c_str());
    else if (a == "--output") out_file = need();
    else if (a == "--hybrid") hybrid = true;
    else if (a == "--minibatch" || a == "-B") hcfg.mini_batch = std::atoi(need().c_str());
    else if (a == "--thread" || a == "-T") hcfg.thread_cnt = std::atoi(need().c_str());
    else if (a == "--ctx_per_thread" || a == "-C") hcfg.ctx_per_thread = std::atoi(need().c_str());
    else if (a == "--io_backend") {
      if (need() != "memory") {
        std::fprintf(stderr, "only the 'memory' io_backend (pread of the index file) is available\n");
        return 1;
      }
    }
    else if (a == "--ef_search") {
      while (i + 1 < argc && argv[i + 1][0] != '-') efs.push_back(std::atoi(argv[++i]));
    } else usage();
  }
  if (query_file.empty() || cfg.index_file.empty() || cfg.pq_file_prefix.empty() || data_type.empty() || efs.empty())
    usage();
  gustann::DataType dtype;
  if (data_type == "float") dtype = gustann::FLOAT;
  else if (data_type == "uint8") dtype = gustann::UINT8;
  else {
    std::fprintf(stderr, "unrecognized data type %s\n", data_type.c_str());
    return 1;
  }
  for (int ef : efs)
    if (ef < topk) {
      std::fprintf(stderr, "ef_search %d < topk %d\n", ef, topk);
      return 1;
    }

  gustann::GustANN a(dtype, device);
  try {
    if (hybrid) a.init_hybrid(cfg, hcfg);
    else a.init_pure_mem(cfg, use_gpu_mem);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }

  size_t d = 0, nq = 0;
  std::vector<float> q;
  {
    auto raw = read_vecs(query_file, dtype == gustann::UINT8 ? 1 : 4, d, nq);
    q.resize(d * nq);
    if (dtype == gustann::UINT8) {
      for (size_t i = 0; i < q.size(); ++i) q[i] = raw[i];   // u8 queries widened (bin/search_disk.cpp:160-165)
    } else {
      std::memcpy(q.data(), raw.data(), q.size() * 4);
    }
  }
  if (repeat > 1) {   // replicate the query set (bin/search_disk.cpp:172-183)
    std::vector<float> r(q.size() * repeat);
    for (int i = 0; i < repeat; ++i) std::memcpy(&r[i * q.size()], q.data(), q.size() * 4);
    q.swap(r);
    nq *= repeat;
  }
  std::unique_ptr<int[]> nns(new int[nq * topk]);
  std::unique_ptr<float[]> dis(new float[nq * topk]);
  std::unique_ptr<int[]> found(new int[nq]);

  std::vector<int> gt;
  size_t gt_d = 0, gt_n = 0;
  if (!gt_file.empty()) {
    auto raw = read_vecs(gt_file, 4, gt_d, gt_n);
    gt.resize(gt_d * gt_n);
    std::memcpy(gt.data(), raw.data(), gt.size() * 4);
  }

  try {
    if (efs.size() == 1) {
      a.search(q.data(), static_cast<int>(nq), topk, efs[0], nns.get(), dis.get(), found.get());
      for (size_t i = 0; i < 5 && i < nq; ++i) {
        for (int j = 0; j < 5 && j < topk; ++j) std::printf("%lf(%d)\t", dis[i * topk + j], nns[i * topk + j]);
        std::printf("\n");
      }
      if (!gt.empty()) {
        const double r = calc_recall(nns.get(), gt.data(), gt_n, gt_d, topk);
        std::printf("Recall @ %d: %lf\n", topk, r);
        std::printf("[REPORT] RECALL: %lf\n", r);
      }
    } else {
      struct Row { int ef; double qps, recall; };
      std::vector<Row> rows;
      for (int ef : efs) {
        gustann::GustANNStats st;
        a.search(q.data(), static_cast<int>(nq), topk, ef, nns.get(), dis.get(), found.get(), &st);
        const bool rec = !gt.empty() && topk <= static_cast<int>(gt_d);
        rows.push_back({ef, nq / st.run_time, rec ? calc_recall(nns.get(), gt.data(), gt_n, gt_d, topk) : -1.0});
      }
      const std::string rh = gt.empty() ? "Recall" : "Recall@" + std::to_string(topk);
      std::printf("\n%-12s %-18s %-18s %-18s\n", "L", "Run Time (s)", "QPS", rh.c_str());
      std::printf("%-12s %-18s %-18s %-18s\n", "------------", "------------------", "------------------",
                  "------------------");
      for (const auto& r : rows) {
        if (r.recall >= 0) std::printf("%-12d %-18.6f %-18.2f %-18.6f\n", r.ef, nq / r.qps, r.qps, r.recall);
        else std::printf("%-12d %-18.6f %-18.2f %-18s\n", r.ef, nq / r.qps, r.qps, "N/A");
      }
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
  if (!out_file.empty()) {
    FILE* f = std::fopen(out_file.c_str(), "wb");
    const int32_t head[2] = {static_cast<int32_t>(nq), topk};
    const bool ok = f && std::fwrite(head, 4, 2, f) == 2 &&
                    std::fwrite(nns.get(), 4, nq * topk, f) == nq * static_cast<size_t>(topk);
    if (f) std::fclose(f);
    if (!ok) {
      std::fprintf(stderr, "cannot write %s\n", out_file.c_str());
      return 1;
    }
  }
  return 0;
}
