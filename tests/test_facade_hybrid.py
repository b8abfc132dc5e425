"""The C++ facade's hybrid search loop (include/gustann.hpp, search_hybrid),
on the CPU, against a fake of the C ABI's hop calls.

The fake gives every query a fixed number of hops and a node id per hop; its
page reader writes the node id into the page, and its hop step fails on a
page that does not hold the node the query asked for. So the loop must hand
each batch the pages of its own latest requests, whether one mini-batch is in
flight or several (ctx_per_thread), with a second thread reading one batch's
pages while another batch steps. Results must land in every query's own row,
and a failed page read must surface as an exception with every batch freed.
"""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = r"""
#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>
#include "gann.h"

struct gann_handle { int dim; };
struct gann_hop_batch { std::vector<int> q, left, step; };
static std::atomic<int> g_live{0};
static int node_of(const gann_hop_batch* b, size_t i) { return 1000 * b->q[i] + b->step[i]; }
static int hops_of(int q) { return 1 + q % 7; }

extern "C" {
int gann_open(const gann_config*, gann_handle** out) { *out = new gann_handle{4}; return GANN_OK; }
int gann_close(gann_handle* h) { delete h; return GANN_OK; }
int gann_search(gann_handle*, const float*, int64_t, int32_t, int32_t, int32_t*, float*, int32_t*, gann_stats*) {
  return GANN_EUNSUPPORTED;
}
const char* gann_last_error(void) { return "fake failure"; }
int gann_index_info(const gann_handle* h, gann_info* out) {
  std::memset(out, 0, sizeof *out);
  out->dim = h->dim;
  out->nodes_per_page = 1;
  return GANN_OK;
}
int gann_hop_begin(gann_handle* h, const float* q, int64_t nq, int32_t, int32_t, gann_hop_batch** out) {
  auto* b = new gann_hop_batch;
  for (int64_t i = 0; i < nq; ++i) {
    const int v = static_cast<int>(q[i * h->dim]);
    b->q.push_back(v);
    b->left.push_back(hops_of(v));
    b->step.push_back(0);
  }
  ++g_live;
  *out = b;
  return GANN_OK;
}
int gann_hop_requests(gann_hop_batch* b, int32_t* ids, int64_t* active) {
  *active = 0;
  for (size_t i = 0; i < b->q.size(); ++i) {
    ids[i] = b->left[i] > 0 ? node_of(b, i) : -1;
    *active += ids[i] >= 0;
  }
  return GANN_OK;
}
int gann_read_pages(const char*, const int32_t* ids, int64_t n, int32_t, void* pages, int32_t) {
  std::this_thread::sleep_for(std::chrono::microseconds(200));
  for (int64_t i = 0; i < n; ++i) {
    if (ids[i] == 13 * 1000 + 2) return GANN_EIO;          // query value 13, third hop
    if (ids[i] >= 0) std::memcpy(static_cast<char*>(pages) + i * 4096, &ids[i], 4);
  }
  return GANN_OK;
}
int gann_hop_step(gann_hop_batch* b, const void* pages) {
  std::this_thread::sleep_for(std::chrono::microseconds(200));
  for (size_t i = 0; i < b->q.size(); ++i) {
    if (b->left[i] <= 0) continue;
    int got;
    std::memcpy(&got, static_cast<const char*>(pages) + i * 4096, 4);
    if (got != node_of(b, i)) return GANN_EINVAL;           // a page of another request
    --b->left[i];
    ++b->step[i];
  }
  return GANN_OK;
}
int gann_hop_finish(gann_hop_batch* b, int32_t* nns, float* dist, int32_t* found) {
  for (size_t i = 0; i < b->q.size(); ++i) {
    nns[2 * i] = b->q[i];
    nns[2 * i + 1] = b->step[i];
    dist[2 * i] = dist[2 * i + 1] = 0.f;
    found[i] = 2;
  }
  return GANN_OK;
}
int gann_hop_free(gann_hop_batch* b) { delete b; --g_live; return GANN_OK; }
int fake_live_batches() { return g_live.load(); }
}
"""

DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "gustann.hpp"
extern "C" int fake_live_batches();

int main(int argc, char** argv) {
  const int k = std::atoi(argv[1]), nq = std::atoi(argv[2]), batch = std::atoi(argv[3]);
  const int base = argc > 4 ? std::atoi(argv[4]) : 0;
  std::vector<float> q(static_cast<size_t>(nq) * 4, 0.f);
  for (int i = 0; i < nq; ++i) q[static_cast<size_t>(i) * 4] = static_cast<float>(base + i);
  gustann::GustANN g(gustann::FLOAT);
  gustann::HybridExecutorConfig hc;
  hc.mini_batch = batch;
  hc.thread_cnt = 2;
  hc.ctx_per_thread = k;
  gustann::GustANNConfig cfg;
  cfg.index_file = "unused";
  g.init_hybrid(cfg, hc);
  std::vector<int> nns(static_cast<size_t>(nq) * 2, -1), found(nq, -1);
  std::vector<float> dist(static_cast<size_t>(nq) * 2, -1.f);
  gustann::GustANNStats st;
  try {
    g.search(q.data(), nq, 2, 4, nns.data(), dist.data(), found.data(), &st);
  } catch (const std::exception& e) {
    std::printf("error %s live %d\n", e.what(), fake_live_batches());
    return 3;
  }
  for (int i = 0; i < nq; ++i) std::printf("%d %d %d\n", nns[2 * i], nns[2 * i + 1], found[i]);
  std::printf("hops %lld live %d\n", st.hops, fake_live_batches());
  return 0;
}
"""


@pytest.fixture(scope="module")
def prog(tmp_path_factory):
    d = tmp_path_factory.mktemp("facade")
    (d / "fake.cpp").write_text(FAKE)
    (d / "driver.cpp").write_text(DRIVER)
    exe = d / "driver"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), str(d / "driver.cpp"),
                    str(d / "fake.cpp"), "-o", str(exe), "-pthread"], check=True)
    return str(exe)


@pytest.mark.parametrize("k,nq,batch", [(0, 37, 8), (1, 37, 8), (2, 37, 8), (3, 100, 7), (5, 12, 5), (4, 9, 100)])
def test_hybrid_loop_hands_each_batch_its_own_pages(prog, k, nq, batch):
    # query values 0.. avoid 13 except where the failure case wants it
    r = subprocess.run([prog, str(k), str(nq), str(batch), "20"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.split("\n")
    rows = np.array([[int(x) for x in ln.split()] for ln in lines[:nq]])
    v = 20 + np.arange(nq)
    np.testing.assert_array_equal(rows[:, 0], v)               # every query's own row
    np.testing.assert_array_equal(rows[:, 1], 1 + v % 7)       # all its hops, in order
    np.testing.assert_array_equal(rows[:, 2], 2)
    tail = lines[nq].split()
    assert tail[0] == "hops" and tail[2] == "live" and tail[3] == "0"


@pytest.mark.parametrize("k", [1, 3])
def test_failed_page_read_raises_and_frees_every_batch(prog, k):
    r = subprocess.run([prog, str(k), "40", "6", "0"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 3, r.stdout + r.stderr
    assert r.stdout.startswith("error gann error") and r.stdout.rstrip().endswith("live 0"), r.stdout
