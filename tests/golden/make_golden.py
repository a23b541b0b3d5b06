#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the reference source tree.

The reference (Jayluci4/nova-wino-amd) ships no golden vectors and its kernels
need hipcc/ROCm/rocBLAS, which this machine does not have.  What it does ship
that runs here, and what this script turns into fixtures:

* ``nova_matrices.json`` -- the host tables nova_A_h / nova_B_h / nova_G_h,
  parsed as text from ``csrc/nova_winograd.hip:68-97``.
* ``tiling.json`` -- outputs of the reference's own ``compute_tiling``
  (``csrc/nova_winograd.hip:617-631``, plain C with no HIP dependency): the
  function's text is cut out of the .hip file, compiled with gcc next to a small
  driver written here, and run over a grid of (H, W, pad).
* ``known_answers.json`` -- numbers the reference publishes for this path
  (FP16 relative error, test tolerances), with file:line.

Usage:  python tests/golden/make_golden.py <reference checkout>
        (or set NOVA_REFERENCE_DIR)
Nothing in the test suite runs this; the fixtures it wrote are committed.
"""

import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def parse_table(src, name):
    m = re.search(r"static const float %s\[(\d+)\]\[(\d+)\]\s*=\s*\{(.*?)\};" % name, src, re.S)
    if not m:
        raise RuntimeError(f"table {name} not found")
    rows, cols = int(m.group(1)), int(m.group(2))
    nums = [float(t.rstrip("f")) for t in re.findall(r"-?\d+\.\d+f?", m.group(3))]
    if len(nums) != rows * cols:
        raise RuntimeError(f"table {name}: expected {rows * cols} numbers, got {len(nums)}")
    return [nums[r * cols:(r + 1) * cols] for r in range(rows)]


def extract_function(src, signature):
    start = src.index(signature)
    depth, i = 0, src.index("{", start)
    for j in range(i, len(src)):
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return src[start:j + 1]
    raise RuntimeError("unbalanced braces")


DRIVER = r"""
#include <stdio.h>
int main(void) {
  int pads[3] = {0, 1, 2};
  printf("[");
  int first = 1;
  for (int pi = 0; pi < 3; ++pi)
    for (int H = 1; H <= 260; ++H) {
      int W = (H * 7) % 253 + 1;
      int nh, nw, Ho, Wo;
      if (H + 2 * pads[pi] - 2 <= 0 || W + 2 * pads[pi] - 2 <= 0) continue;
      compute_tiling(H, W, pads[pi], &nh, &nw, &Ho, &Wo);
      printf("%s[%d,%d,%d,%d,%d,%d,%d]", first ? "" : ",", H, W, pads[pi], nh, nw, Ho, Wo);
      first = 0;
    }
  printf("]\n");
  return 0;
}
"""


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NOVA_REFERENCE_DIR")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set NOVA_REFERENCE_DIR)")
    path = os.path.join(ref, "csrc", "nova_winograd.hip")
    src = open(path).read()

    mats = {
        "source": "csrc/nova_winograd.hip:68-97",
        "A": parse_table(src, "nova_A_h"),
        "B": parse_table(src, "nova_B_h"),
        "G": parse_table(src, "nova_G_h"),
    }
    with open(os.path.join(HERE, "nova_matrices.json"), "w") as f:
        json.dump(mats, f, indent=1)

    fn = extract_function(src, "void compute_tiling(int H, int W, int pad")
    with tempfile.TemporaryDirectory() as d:
        c_path = os.path.join(d, "tiling.c")
        with open(c_path, "w") as f:
            f.write(fn + "\n" + DRIVER)
        exe = os.path.join(d, "tiling")
        subprocess.check_call(["gcc", "-O1", "-x", "c", c_path, "-o", exe])
        rows = json.loads(subprocess.check_output([exe]).decode())
    with open(os.path.join(HERE, "tiling.json"), "w") as f:
        json.dump({"source": "csrc/nova_winograd.hip:617-631 compiled with gcc",
                   "columns": ["H", "W", "pad", "nh", "nw", "H_out", "W_out"],
                   "rows": rows}, f)

    known = {
        "fp16_rel_error_vs_fp32_direct": {
            "value": 0.052,
            "source": "docs/report/main.tex:217,221; docs/report/generate_figures.py:121",
        },
        "test_rel_l2_tolerance": {"value": 0.06, "source": "tests/test_correctness.py:84"},
        "backward_grad_input_tolerance": {"value": 0.10, "source": "tests/test_correctness.py:164"},
        "backward_grad_weight_tolerance": {"value": 0.15, "source": "tests/test_correctness.py:165"},
        "resnet50_eligible_convs": {"value": 13, "source": "docs/report/main.tex:185"},
    }
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
