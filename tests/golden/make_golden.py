#!/usr/bin/env python3
"""Regenerate the committed golden fixtures from the reference itself.

Needs the reference source tree, given as the first argument or in the
environment variable TRIA_REF_SRC (there is no default), and the compiled
reference library (`make -C oracle ref REF=<reference tree>`).  Outputs, all under tests/golden/:

  synth_l2h8kv4.tria          seeded TRIA v2 stats (2 layers, 8 heads, 4 kv, hd 128,
                              theta 1e6, layer scales 0.9 / 1.1)
  kat_single_synth_L1H3.bin   reference triattention_export_test.py on the synthetic
                              stats (layer 1, head 3): raw single-head scores
  kat_single_qwen3-8b_L3H5.bin  same exporter on the shipped qwen3-8b stats
  kat_gqa_synth_L1KV2.bin     reference triattention_export_test_gqa.py (layer 1,
                              kv-head 2): z-normalised (unbiased std) GQA max
  refc_synth_L{l}KV{h}_n{n}.bin  the compiled reference C tria_score_kv_head on
                              seeded keys; layout (little-endian):
                              i32 fc, n, cur_pos, layer, kv_head; i32 key_pos[n];
                              f32 k_re[n*fc]; f32 k_im[n*fc]; f32 expected[n]

Run:  python tests/golden/make_golden.py <reference tree>
"""
import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "triattention-ggml_b200"))
import workloads  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TRIA_REF_SRC", "")
if not REF or not os.path.exists(os.path.join(REF, "triattention.c")):
    sys.exit("make_golden.py: give the reference source tree (the directory holding triattention.c) "
             "as the first argument or in TRIA_REF_SRC")


def run_exporter(script, stats, out, layer, head):
    cmd = [sys.executable, os.path.join(REF, script), stats, out, str(layer), str(head)]
    subprocess.run(cmd, check=True, cwd=REF)


def refc_case(lib, stats_path, layer, kv_head, n, cur_pos, seed, pos_mode):
    st = lib.tria_load(stats_path.encode())
    assert st
    fc = 64
    k = workloads.fp32_keys(n, 2 * fc, seed=seed)[0]
    k_re, k_im = workloads.split_halves(k)
    rng = np.random.default_rng(seed + 1)
    if pos_mode == "dense":
        key_pos = np.arange(n, dtype=np.int32) + (cur_pos - n)
    else:   # sorted distinct positions spread over [0, cur_pos)
        key_pos = np.sort(rng.choice(cur_pos, size=n, replace=False)).astype(np.int32)
    out = np.zeros(n, np.float32)
    P = ctypes.POINTER(ctypes.c_float)
    lib.tria_score_kv_head(st, k_re.ctypes.data_as(P), k_im.ctypes.data_as(P),
                           key_pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                           cur_pos, n, layer, kv_head, out.ctypes.data_as(P))
    lib.tria_free(st)
    name = os.path.join(HERE, f"refc_synth_L{layer}KV{kv_head}_n{n}.bin")
    with open(name, "wb") as f:
        f.write(np.array([fc, n, cur_pos, layer, kv_head], "<i4").tobytes())
        f.write(key_pos.astype("<i4").tobytes())
        f.write(k_re.astype("<f4").tobytes())
        f.write(k_im.astype("<f4").tobytes())
        f.write(out.astype("<f4").tobytes())
    return name


def main():
    stats = os.path.join(HERE, "synth_l2h8kv4.tria")
    workloads.write_tria(stats, 2, 8, 4, 128, rope_theta=1e6,
                         scales=np.array([0.9, 1.1], np.float32), seed=7)
    run_exporter("triattention_export_test.py", stats,
                 os.path.join(HERE, "kat_single_synth_L1H3.bin"), 1, 3)
    run_exporter("triattention_export_test.py", os.path.join(REF, "stats", "qwen3-8b.bin"),
                 os.path.join(HERE, "kat_single_qwen3-8b_L3H5.bin"), 3, 5)
    run_exporter("triattention_export_test_gqa.py", stats,
                 os.path.join(HERE, "kat_gqa_synth_L1KV2.bin"), 1, 2)

    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libtria_ref.so"))
    lib.tria_load.restype = ctypes.c_void_p
    lib.tria_load.argtypes = [ctypes.c_char_p]
    lib.tria_free.argtypes = [ctypes.c_void_p]
    lib.tria_score_kv_head.argtypes = [ctypes.c_void_p] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    refc_case(lib, stats, 1, 2, 300, 70000, 11, "spread")
    refc_case(lib, stats, 0, 1, 512, 512, 12, "dense")


if __name__ == "__main__":
    main()
