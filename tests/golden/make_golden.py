"""Generate the golden fixtures in this directory.

Run from the repository root in a container that has the reference checkout:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

What it writes:

* ``ref_gmm_golden.npz`` -- for every case in ``cases.py``, sampled output rows
  of the REFERENCE'S OWN oracle ``ref_gmm`` (reference
  ``tests/test_forward.py:8-15``), imported from the reference checkout and
  run on CPU tensors in the case dtype.  Values are stored as raw bit
  patterns (uint32 for fp32, uint16 for bf16/fp16).
* ``config_batch_sizes.json`` -- the frozen ``batch_sizes`` of the five
  workload configurations (``gmm_b200.configs.batch_sizes_for``).

The reference package cannot be imported without its compiled extension
because it registers a fake impl for an op that the extension defines; the
script defines that op's schema first (no implementation), which is all the
package import needs.  Nothing else of the reference is executed.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(1, ROOT)

from cases import all_cases, make_case_inputs, sample_rows  # noqa: E402


def load_reference_ref_gmm(ref_root: str):
    lib = torch.library.Library("hopper_gmm_fwd", "DEF")  # noqa: F841 (kept alive below)
    lib.define("gmm(Tensor A, Tensor B, Tensor batch_sizes, bool trans_b) -> Tensor")
    sys.path.insert(0, ref_root)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)
        spec = importlib.util.spec_from_file_location(
            "reference_test_forward", os.path.join(ref_root, "tests", "test_forward.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    mod._keepalive_lib = lib
    return mod.ref_gmm


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.contiguous().view(torch.int32).numpy().view(np.uint32)
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref_gmm = load_reference_ref_gmm(args.reference)

    out = {}
    meta = []
    for case in all_cases():
        a, b, bs = make_case_inputs(case)
        d = ref_gmm(a, b, bs, trans_b=case["trans_b"])
        rows = sample_rows(case["bs"])
        out[case["name"] + "__rows"] = np.asarray(rows, dtype=np.int64)
        out[case["name"] + "__out"] = bits(d[rows])
        meta.append(case)
        print(f"{case['name']:34s} T={sum(case['bs']):5d} rows={len(rows):3d} dtype={case['dtype']}")
    out["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "ref_gmm_golden.npz"), **out)

    from gmm_b200.configs import CONFIGS, batch_sizes_for
    frozen = {str(c): batch_sizes_for(cfg).tolist() for c, cfg in CONFIGS.items()}
    with open(os.path.join(HERE, "config_batch_sizes.json"), "w") as f:
        json.dump(frozen, f)
        f.write("\n")
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
