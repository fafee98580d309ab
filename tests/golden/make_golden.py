"""Generate the golden vectors under tests/golden/ by running the REFERENCE
library (oracle/_ref/libcusort_ref.so: libcusort.cuh compiled for sm_100a,
unmodified) on a B200.

Usage (on a GPU machine, with oracle/_ref built):
    python tests/golden/make_golden.py <out_dir>
then copy <out_dir>/* into tests/golden/.  Each case stores the seeded input
and the reference's output (in/out-pointer API); tests/test_oracle.py checks
the CPU oracle against them, which pins the oracle to the reference.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from tests import datagen as D  # noqa: E402
from tests.gpu_helpers import run_ref  # noqa: E402


def cases():
    out = []
    for i, kt in enumerate(D.KEY_TYPES):
        for desc in (False, True):
            n = 3001 + 97 * i
            keys = D.special_floats(kt, n, seed=100 + i, frac=0.01) if kt.startswith("f") else \
                D.uniform_bits(kt, n, seed=100 + i)
            out.append((f"{kt}_{'desc' if desc else 'asc'}_pairs_u32", kt, keys, D.values_for(n, 4), 0,
                        8 * keys.dtype.itemsize, desc))
    out.append(("config1_u32_keys_4096", "u32", D.uniform_bits("u32", 4096, seed=1), None, 0, 32, False))
    out.append(("i32_low_entropy", "i32", D.low_entropy("i32", 5000, seed=3), D.values_for(5000, 4), 0, 32,
                False))
    out.append(("u32_zipf_bits0_20", "u32", D.zipf_table("u32", 5000, seed=6), D.values_for(5000, 4), 0, 20,
                False))
    out.append(("f32_bits3_29_desc", "f32", D.special_floats("f32", 4000, seed=7), D.values_for(4000, 4), 3, 29,
                True))
    out.append(("i64_bits17_61", "i64", D.uniform_bits("i64", 4000, seed=8), D.values_for(4000, 8), 17, 61,
                False))
    out.append(("f64_bits40_64_v16", "f64", D.special_floats("f64", 3000, seed=9), D.values_for(3000, 16), 40, 64,
                False))
    out.append(("u8_v1", "u8", D.uniform_bits("u8", 5000, seed=10), D.values_for(5000, 1), 0, 8, False))
    out.append(("i16_v2_desc", "i16", D.uniform_bits("i16", 5000, seed=11), D.values_for(5000, 2), 0, 16, True))
    out.append(("u16_bits4_12", "u16", D.uniform_bits("u16", 5000, seed=12), D.values_for(5000, 4), 4, 12,
                False))
    return out


def main(out_dir: str) -> None:
    od = Path(out_dir)
    od.mkdir(parents=True, exist_ok=True)
    index = []
    for name, kt, keys, vals, b, e, desc in cases():
        ko, vo, _ = run_ref(kt, keys, vals, b, e, desc, api="raw")
        arrays = {"keys_in": keys, "keys_out": ko}
        if vals is not None:
            arrays["values_in"] = vals
            arrays["values_out"] = vo
        np.savez_compressed(od / f"{name}.npz", **arrays)
        index.append({"name": name, "file": f"{name}.npz", "key_type": kt, "begin_bit": b, "end_bit": e,
                      "descending": desc, "n": int(keys.shape[0]),
                      "value_bytes": 0 if vals is None else int(vals.nbytes // keys.shape[0])})
    (od / "index.json").write_text(json.dumps({
        "generator": "tests/golden/make_golden.py",
        "reference": "IlyaGrebnov/libcusort 1.0.1 libcusort.cuh, nvcc 12.9 -arch sm_100a, in/out-pointer API",
        "cases": index}, indent=1))
    print(f"wrote {len(index)} cases to {od}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(ROOT / "tests" / "golden"))
