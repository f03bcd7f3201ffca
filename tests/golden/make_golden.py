#!/usr/bin/env python3
"""Regenerate the golden fixtures in this folder from the reference tree.

The fixtures are the reference's own small binary test inputs for the Q8 and
bf16 GEMM paths, copied byte for byte, plus `golden.json`, which records the
outputs the reference's reports give for them. The parity tests read only this
folder, so they run where the reference tree is absent.

Usage: python tests/golden/make_golden.py <path-to-reference-root>

Sources (paths inside the shouzugzs-AI/Sparrow tree):
  examples/p13/q8_{a.f32,w.i8,scale.f32}   written by tools/p13_q8_check.py:97-99,
                                            expected [-1,-1] (tools/p13_q8_check.py:45-50)
  sparrow/examples/int8_bins/               written by sparrow/tools/gen_int8.py:58-95
  sparrow/examples/int8_bad_bins/           same set with a_scale[0] += 2^-6 (gen_int8.py:96-100)
  sparrow/examples/int8_naive_bins/         scale = max|row|/127 (gen_int8.py:84-93)
  sparrow/examples/bf16_bins_{bf16,f32}/    written by sparrow/tools/gen_bf16.py
  sparrow/examples/e2e_bins/e2e_tiny.vmb    a whole .vmb program (7 f32 constants, 11 slots, an OP_GEMM),
                                            with its constants' .bin files and the .args manifest
Recorded outputs: sparrow/REPORT_V015.md:443-446 (criteria 1-4 of
sparrow/tools/int8_ab.ps1), printed with the engine's truncating print_f32
(core/src/interp.rs:2416-2473).
"""
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

COPY = {
    "p13": ("examples/p13", ["q8_a.f32", "q8_w.i8", "q8_scale.f32"]),
    "int8_bins": ("sparrow/examples/int8_bins", None),
    "int8_bad_bins": ("sparrow/examples/int8_bad_bins", None),
    "int8_naive_bins": ("sparrow/examples/int8_naive_bins", None),
    "bf16_bins_bf16": ("sparrow/examples/bf16_bins_bf16", ["LINEAR_W.bin", "EMBED_E.bin"]),
    "bf16_bins_f32": ("sparrow/examples/bf16_bins_f32", ["LINEAR_W.bin", "EMBED_E.bin"]),
    "e2e_tiny": ("sparrow/examples/e2e_bins", ["e2e_tiny.vmb", "e2e_tiny.args", "tiny_in.bin", "EMBED_E.bin",
                                               "SPARSE_off.bin", "SPARSE_src.bin", "SPARSE_W.bin", "LINEAR_W.bin",
                                               "LINEAR_b.bin"]),
}

GOLDEN = {
    "p13_q8": {
        "source": "tools/p13_q8_check.py:45-50",
        "a_shape": [1, 4], "w_shape": [2, 4],
        "expected": [-1.0, -1.0],
    },
    "int8_one_k1": {
        "source": "sparrow/REPORT_V015.md:443 (criterion 1: f32 and int8 print identically)",
        "model": "o = linear(in=1,out=4) + bias; input i8o_in.bin",
        "printed": "0.881869 -0.907158 -0.010653 2.102990",
    },
    "int8_two_k4_exact": {
        "source": "sparrow/REPORT_V015.md:444 (criterion 2: max diff <= 1e-4, measured 0)",
        "model": "b(a(x)), each linear + bias; input i8t_in.bin",
        "max_diff_bound": 1e-4, "measured": 0.0,
    },
    "int8_two_bad_scale": {
        "source": "sparrow/REPORT_V015.md:445 (criterion 3: can-fail)",
        "max_diff": 0.607249,
    },
    "int8_two_naive": {
        "source": "sparrow/REPORT_V015.md:446 (criterion 4: naive quantisation control)",
        "max_diff": 0.009791,
    },
    "bf16_widen": {
        "source": "sparrow/tools/gen_bf16.py (widen(bf16(x)) bit pattern == truncate(x))",
        "files": ["LINEAR_W.bin", "EMBED_E.bin"],
    },
}


def main(ref_root: str) -> None:
    for sub, (src, names) in COPY.items():
        dst = os.path.join(HERE, sub)
        os.makedirs(dst, exist_ok=True)
        srcdir = os.path.join(ref_root, src)
        for fn in names or sorted(os.listdir(srcdir)):
            shutil.copyfile(os.path.join(srcdir, fn), os.path.join(dst, fn))
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(GOLDEN, f, indent=1, sort_keys=True)
        f.write("\n")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
