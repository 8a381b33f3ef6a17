"""Regenerate the committed golden fixtures in this directory.

Run where a reference checkout exists, with the reference checker built by
`make -C oracle REF=<checkout>` (oracle/_ref/libref.so), naming the checkout:

    python tests/golden/make_golden.py --ref <checkout>
    LUNELETTE_REFERENCE=<checkout> python tests/golden/make_golden.py

Outputs (small JSON, committed so the GPU box needs no reference checkout):
  fp8_golden.json   all 256 E4M3FN codes -> FP32 bits, parsed as data from the
                    reference's tests/fp8_golden.h (frozen PyTorch table).
  rope_golden.json  Transformers v5 cos/sin at 5 positions x 4 pair indices,
                    parsed from the reference's tests/rope_golden.h.
  yarn_ref.json     full 128-entry cos/sin bit patterns from the reference's
                    own lunelette_metal_yarn (src/metal_yarn.c) at positions
                    that cover both capacity profiles and the 16384 boundary.
  greedy_ref.json   lunelette_select_greedy (src/generation.c:8-34) answers on
                    seeded vectors with planted ties, signed zeros and NaN/Inf.
"""
import argparse
import ctypes
import json
import os
import re
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
YARN_POSITIONS = [0, 1, 2, 63, 64, 127, 255, 256, 1000, 4095, 4096, 4351,
                  16383, 16384, 16385, 262143]


def parse_fp8(ref):
    text = open(os.path.join(ref, "tests", "fp8_golden.h")).read()
    body = text[text.index("{") + 1:text.rindex("}")]
    words = [int(w, 16) for w in re.findall(r"0x([0-9a-fA-F]+)u", body)]
    assert len(words) == 256
    return words


def parse_rope(ref):
    text = open(os.path.join(ref, "tests", "rope_golden.h")).read()
    body = text[text.index("=") + 1:]
    values = [float(v) for v in re.findall(r"(-?[0-9.]+e[+-][0-9]+)f", body)]
    assert len(values) == 5 * 4 * 2
    table = []
    for p in range(5):
        table.append([[values[(p * 4 + j) * 2], values[(p * 4 + j) * 2 + 1]] for j in range(4)])
    return {"positions": [0, 1, 16383, 16384, 16385], "indices": [1, 24, 40, 63],
            "cos_sin": table, "tolerance": 2e-6,
            "source": "reference tests/rope_golden.h (Transformers v5.0.0 CPU FP32)"}


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def yarn_table(lib):
    lib.lunelette_metal_yarn.argtypes = [ctypes.c_uint32, ctypes.POINTER(ctypes.c_float),
                                         ctypes.POINTER(ctypes.c_float)]
    lib.lunelette_metal_yarn.restype = ctypes.c_int
    out = {}
    for p in YARN_POSITIONS:
        c = (ctypes.c_float * 128)()
        s = (ctypes.c_float * 128)()
        assert lib.lunelette_metal_yarn(p, c, s) == 0
        out[str(p)] = {"cos": [f32_bits(v) for v in c], "sin": [f32_bits(v) for v in s]}
    c = (ctypes.c_float * 128)()
    s = (ctypes.c_float * 128)()
    rejected = lib.lunelette_metal_yarn(262144, c, s)
    return {"positions": YARN_POSITIONS, "tables": out, "rejects_262144": rejected != 0,
            "source": "reference src/metal_yarn.c compiled by oracle/Makefile"}


def greedy_cases(lib):
    lib.lunelette_select_greedy.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                                            ctypes.c_char_p, ctypes.c_size_t]
    lib.lunelette_select_greedy.restype = ctypes.c_int
    rng = np.random.default_rng(20261201)
    cases = []
    for case in range(8):
        v = rng.standard_normal(131072).astype(np.float32)
        plant = {}
        if case == 1:  # exact tie: lowest id wins
            top = float(v.max()) + 1.0
            plant = {"tie": [777, 4242]}
            v[777] = top
            v[4242] = top
        if case == 2:  # signed zeros tie at the top
            v[:] = -1.0
            v[10] = -0.0
            v[5] = 0.0
            plant = {"signed_zero": [5, 10]}
        if case == 3:
            v[99] = np.inf
            plant = {"inf": 99}
        if case == 4:
            v[131071] = np.nan
            plant = {"nan": 131071}
        if case == 5:  # max at the last index
            v[131071] = float(v.max()) + 0.5
        token = ctypes.c_int64(-7)
        err = ctypes.create_string_buffer(256)
        rc = lib.lunelette_select_greedy(v.ctypes.data, ctypes.byref(token), err, 256)
        cases.append({"seed_case": case, "plant": plant, "rc": rc,
                      "token": token.value if rc == 0 else None})
    return {"rng": "numpy default_rng(20261201).standard_normal(131072) per case, float32",
            "cases": cases, "source": "reference src/generation.c:8-34"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("LUNELETTE_REFERENCE"),
                    help="reference checkout (default: $LUNELETTE_REFERENCE)")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(args.ref):
        ap.error("name the reference checkout with --ref or LUNELETTE_REFERENCE")
    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref.so"))
    fp8 = parse_fp8(args.ref)
    lib.st_f8_e4m3_to_f32.argtypes = [ctypes.c_ubyte]
    lib.st_f8_e4m3_to_f32.restype = ctypes.c_float
    decoded = [f32_bits(lib.st_f8_e4m3_to_f32(i)) for i in range(256)]
    for i in range(256):
        if (i & 127) != 127:
            assert decoded[i] == fp8[i], (i, hex(decoded[i]), hex(fp8[i]))
    with open(os.path.join(HERE, "fp8_golden.json"), "w") as f:
        json.dump({"bits": fp8, "nan_codes": [127, 255],
                   "source": "reference tests/fp8_golden.h (frozen PyTorch float8_e4m3fn)"}, f)
    with open(os.path.join(HERE, "rope_golden.json"), "w") as f:
        json.dump(parse_rope(args.ref), f, indent=1)
    with open(os.path.join(HERE, "yarn_ref.json"), "w") as f:
        json.dump(yarn_table(lib), f)
    with open(os.path.join(HERE, "greedy_ref.json"), "w") as f:
        json.dump(greedy_cases(lib), f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
