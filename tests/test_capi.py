"""The C-ABI library loads, exports every symbol include/gann.h declares, and
rejects malformed inputs with status codes -- all without a GPU (files are
parsed before any CUDA call)."""
import os
import re
import shutil
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from gustann_b200 import api, formats
from gustann_b200.api import GustANN, GustANNConfig, GustANNError

HEADER = os.path.join(ROOT, "include", "gann.h")
GOLD = os.path.join(ROOT, "tests", "golden", "g_u8")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(gann_\w+)\s*\(", src, re.M)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert set(syms) == set(api.EXPORTS)


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", api.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (gann_\w+)", out.stdout))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_header_compiles_as_c_and_cpp(tmp_path):
    c = tmp_path / "t.c"
    c.write_text('#include "gann.h"\nint main(void){gann_config c; (void)c; return GANN_OK;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), "-c", str(c),
                    "-o", str(tmp_path / "t.o")], check=True)
    cc = tmp_path / "t.cpp"
    cc.write_text('#include "gustann.hpp"\nint main(){gustann::GustANNConfig c; c.index_file="x"; return 0;}\n')
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), "-c", str(cc),
                    "-o", str(tmp_path / "t2.o")], check=True)


def test_facade_program_links_against_the_library(tmp_path):
    """A driver written against gustann::GustANN (in-HBM and hybrid modes)
    compiles and links against libgann.so (not run: no GPU here)."""
    src = tmp_path / "drv.cpp"
    src.write_text(
        '#include "gustann.hpp"\n'
        "int main(int argc, char** argv) {\n"
        "  gustann::GustANN a(gustann::FLOAT);\n"
        "  gustann::GustANNConfig c; c.index_file = argv[0]; c.pq_file_prefix = argv[0];\n"
        "  gustann::HybridExecutorConfig h; h.mini_batch = 64; h.thread_cnt = 4;\n"
        "  try { if (argc > 5) a.init_hybrid(c, h); else a.init_pure_mem(c, true); }\n"
        "  catch (const std::exception&) { return 0; }\n"
        "  float q[4] = {0}; int n[1]; float d[1]; int f[1]; gustann::GustANNStats st;\n"
        "  a.search(q, 1, 1, 1, n, d, f, &st);\n"
        "  return 0;\n}\n")
    lib_dir = os.path.dirname(api.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), str(src), "-o",
                    str(tmp_path / "drv"), "-L", lib_dir, "-lgann", f"-Wl,-rpath,{lib_dir}"], check=True)


def test_pivot_sample_matches_std_shuffle_semantics():
    a = api.pivot_sample(1000, 100)
    b = api.pivot_sample(1000, 100)
    assert np.array_equal(a, b)
    assert np.all(np.diff(a) > 0) and a.min() >= 0 and a.max() < 1000
    assert np.array_equal(api.pivot_sample(50, 50), np.arange(50))
    with pytest.raises(GustANNError):
        api.pivot_sample(10, 11)


def _open_expect(cfg, code):
    g = GustANN(formats.UINT8)
    with pytest.raises(GustANNError) as e:
        g.init_pure_mem(cfg, True)
    assert e.value.code == code, str(e.value)


def _copy_golden(tmp_path):
    d = tmp_path / "idx"
    shutil.copytree(GOLD, d)
    return formats.index_paths(str(d))


def test_missing_files(tmp_path):
    p = _copy_golden(tmp_path)
    _open_expect(GustANNConfig(str(tmp_path / "nope"), p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EIO)
    _open_expect(GustANNConfig(p["index_file"], str(tmp_path / "nope"), p["nav_graph_prefix"]), api.GANN_EIO)
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], str(tmp_path / "nope")), api.GANN_EIO)


def test_wrong_dtype_is_rejected(tmp_path):
    p = _copy_golden(tmp_path)
    g = GustANN(formats.FLOAT)
    with pytest.raises(GustANNError) as e:
        g.init_pure_mem(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), True)
    assert e.value.code == api.GANN_EINVAL


def test_corrupt_header(tmp_path):
    p = _copy_golden(tmp_path)
    with open(p["index_file"], "r+b") as f:
        f.seek(8)
        f.write(struct.pack("<Q", 0))          # zero nodes
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EINVAL)


def test_truncated_index(tmp_path):
    p = _copy_golden(tmp_path)
    size = os.path.getsize(p["index_file"])
    with open(p["index_file"], "r+b") as f:
        f.truncate(size - 4096)
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EIO)


def test_bad_neighbour_id(tmp_path):
    """Out-of-range ids are caught while records are re-laid out; that step runs
    after the CUDA check, so here (no GPU) the CPU parser is exercised directly
    on the record layout instead."""
    p = _copy_golden(tmp_path)
    lay, vec, deg, nbrs = formats.read_disk_index(p["index_file"], formats.UINT8)
    assert np.all(nbrs[np.arange(lay.max_m0)[None, :] < deg[:, None]] < lay.num_data)


def test_pq_chunk_offsets_must_cover_dim(tmp_path):
    p = _copy_golden(tmp_path)
    piv, cen, offs, codes = formats.read_pq(p["pq_file_prefix"])
    bad = offs.copy()
    bad[-1] -= 1
    formats.write_pq(p["pq_file_prefix"], piv, cen, bad, codes)
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EINVAL)


def test_pq_row_count_must_match(tmp_path):
    p = _copy_golden(tmp_path)
    piv, cen, offs, codes = formats.read_pq(p["pq_file_prefix"])
    formats.write_pq(p["pq_file_prefix"], piv, cen, offs, codes[:-1])
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EINVAL)


def test_nav_bad_ids(tmp_path):
    p = _copy_golden(tmp_path)
    vec, adj, start, ids = formats.read_nav(p["nav_graph_prefix"], formats.UINT8)
    ids2 = ids.copy()
    ids2[0] = 10 ** 8
    deg = (adj >= 0).sum(1)
    formats.write_nav(p["nav_graph_prefix"], vec, ids2, adj, deg, start, max_degree=adj.shape[1])
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EINVAL)
    adj2 = adj.copy()
    adj2[3, 0] = len(ids) + 5
    formats.write_nav(p["nav_graph_prefix"], vec, ids, adj2, deg, start, max_degree=adj.shape[1])
    _open_expect(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), api.GANN_EINVAL)


def test_legacy_pq_layout_is_parsed(tmp_path):
    """nr == 5 pivot tables (PipeANN/older DiskANN) put chunk offsets in slot 3."""
    p = _copy_golden(tmp_path)
    piv, cen, offs, codes = formats.read_pq(p["pq_file_prefix"])
    formats.write_pq(p["pq_file_prefix"], piv, cen, offs, codes, legacy=True)
    piv2, cen2, offs2, codes2 = formats.read_pq(p["pq_file_prefix"])
    assert np.array_equal(offs2, offs)
    g = GustANN(formats.UINT8)
    with pytest.raises(GustANNError) as e:      # parses fine; fails only at the CUDA step
        g.init_pure_mem(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), True)
    assert e.value.code in (api.GANN_ECUDA, api.GANN_EINVAL) or e.value.code == api.GANN_OK


def test_use_before_init():
    with pytest.raises(GustANNError) as e:
        GustANN(formats.UINT8).query(np.zeros((1, 4), np.float32), 1, 1)
    assert e.value.code == api.GANN_ESTATE


def test_hybrid_open_parses_files_first(tmp_path):
    """init_hybrid (records left on storage) validates the files like init_pure_mem."""
    p = _copy_golden(tmp_path)
    g = GustANN(formats.UINT8)
    with pytest.raises(GustANNError) as e:
        g.init_hybrid(GustANNConfig(str(tmp_path / "nope"), p["pq_file_prefix"], p["nav_graph_prefix"]))
    assert e.value.code == api.GANN_EIO


def test_cli_usage_and_errors():
    cli = os.path.join(ROOT, "gustann_b200", "_lib", "search_mem")
    r = subprocess.run([cli], capture_output=True, text=True)
    assert r.returncode != 0 and "usage" in r.stderr
    r = subprocess.run([cli, "--query", "x", "--index", "/nonexistent", "--pq_data", "p", "--data_type", "uint8",
                        "--ef_search", "10", "--topk", "10"], capture_output=True, text=True)
    assert r.returncode != 0 and "cannot open index file" in r.stderr


def test_config_struct_matches_the_header(tmp_path):
    """ctypes' gann_config has the C struct's size and field offsets."""
    import ctypes
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "gann.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu\\n", sizeof(gann_config), offsetof(gann_config, layout),'
                   ' offsetof(gann_config, part_count), offsetof(gann_config, part_index)); return 0;}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    C = api._Config
    assert got == [ctypes.sizeof(C), C.layout.offset, C.part_count.offset, C.part_index.offset]


def test_split_record_options_are_validated(tmp_path):
    p = _copy_golden(tmp_path)
    cfg = GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"])
    for count, index, gpu_mem, code in [(9, 0, True, api.GANN_EINVAL), (-1, 0, True, api.GANN_EINVAL),
                                        (2, 2, True, api.GANN_EINVAL), (3, -2, True, api.GANN_EINVAL),
                                        (2, 0, False, api.GANN_EUNSUPPORTED)]:
        g = GustANN(formats.UINT8)
        with pytest.raises(GustANNError) as e:
            g.init_pure_mem(cfg, gpu_mem, part_count=count, part_index=index)
        assert e.value.code == code, (count, index, gpu_mem, str(e.value))


def test_part_calls_reject_bad_arguments():
    blob = b"\0" * api.PART_BLOB_BYTES
    assert api.lib.gann_part_export(None, None, 0) == api.GANN_EINVAL
    assert api.lib.gann_part_attach(None, 0, blob, len(blob)) == api.GANN_EINVAL


def test_check_recall_tool(tmp_path):
    """check_recall (bin/check_recall.cpp:11-32): recall of a bin result file
    against an ivecs ground truth, and its errors."""
    import subprocess
    from gustann_b200 import build as nb
    tool = nb.build_check()
    gt = np.array([[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12]], np.int32)
    formats.write_vecs(str(tmp_path / "gt.ivecs"), gt)
    res = np.array([[2, 1, 0], [5, 5, 9], [0, 0, 0]], np.int32)
    formats.write_bin(str(tmp_path / "out.bin"), res)
    r = subprocess.run([tool, str(tmp_path / "out.bin"), str(tmp_path / "gt.ivecs")], capture_output=True, text=True)
    assert r.returncode == 0
    # row 0: {2,1} in top-3 {1,2,3}; row 1: 5 twice (each counts); row 2: none
    assert r.stdout.strip() == f"Recall @ 3: {4 / 9:.6f}"
    formats.write_bin(str(tmp_path / "short.bin"), res[:2])
    r = subprocess.run([tool, str(tmp_path / "short.bin"), str(tmp_path / "gt.ivecs")], capture_output=True, text=True)
    assert r.returncode != 0 and "NUM mismatch" in r.stdout
    formats.write_bin(str(tmp_path / "wide.bin"), np.zeros((3, 5), np.int32))
    r = subprocess.run([tool, str(tmp_path / "wide.bin"), str(tmp_path / "gt.ivecs")], capture_output=True, text=True)
    assert r.returncode != 0 and "DIM mismatch" in r.stdout
    r = subprocess.run([tool, str(tmp_path / "missing.bin"), str(tmp_path / "gt.ivecs")], capture_output=True, text=True)
    assert r.returncode != 0
