#!/usr/bin/env python3
"""Regenerate the committed golden fixtures from the reference's own Python tooling.

Runs the reference's fixture generator (tests/gen_fixtures.py, which imports tools/qlm.py: the
bit-exact numpy quantizers and the float64 forward_ref) into a scratch directory and copies the
files that pin the hot path into this directory:

  qin.f32 / qin.q8 / qin.q4             quantizer cross-check rows (gen_fixtures.py:72-77)
  {small,odd}_{f32,q8_0,q4_0}.qlm       seeded models + float64 logits on the dequantized weights
  *.ref.f32 / *.reffp.f32 / *.tokens    (.ref) and on the original fp32 weights (.reffp), 20 positions
  l2c_f32.*                             llama2.c-converted model case (gen_fixtures.py:46-54)

Usage:  python tests/golden/make_golden.py REFERENCE_ROOT     (needs the reference checkout;
the committed fixtures are what the tests read, so the GPU box never needs the reference).
"""
import importlib.util
import os
import shutil
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
KEEP = ["qin.f32", "qin.q8", "qin.q4"]
for model in ("small_f32", "small_q8_0", "small_q4_0", "odd_f32", "odd_q8_0", "odd_q4_0", "l2c_f32"):
    KEEP += [f"{model}.qlm", f"{model}.ref.f32", f"{model}.tokens"]
    if not model.endswith("f32"):
        KEEP.append(f"{model}.reffp.f32")


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    spec = importlib.util.spec_from_file_location("gen_fixtures", os.path.join(ref_root, "tests", "gen_fixtures.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    with tempfile.TemporaryDirectory() as tmp:
        gen.main(tmp)
        for name in KEEP:
            shutil.copyfile(os.path.join(tmp, name), os.path.join(HERE, name))
    print(f"wrote {len(KEEP)} golden files to {HERE}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (the reference checkout)")
    main(sys.argv[1])
