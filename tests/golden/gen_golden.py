#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the reference tree.

Needs the reference checkout (--ref, or the BATMOBILE_REF environment variable)
and runs on the CPU:

* cg_l3.json   -- the 34-path / 611-entry CG table parsed from the reference's
                  vendored include/cg_coefficients_l3.cuh:23-792 (BLOCK_INFO,
                  BLOCK_RANGES, ENTRY_INFO, CG_COEFFS).
* sh_ref.npz   -- outputs of the reference's own PyTorch SH code
                  (python/batmobile/autograd.py:97-401, imported with a stub
                  `_batmobile` module): forward for l_max 0..4 and the analytic
                  backward for l_max 3, on seeded random unit vectors plus the
                  axis / diagonal / near-pole vectors of
                  tests/test_spherical_harmonics.py:52-107.
* nl_ref.npz   -- the reference's CPU brute-force neighbour list
                  (tests/test_neighbor_list.cu:30-68, via oracle/_ref) on its own
                  mt19937 positions for N = 100 and 300 at density 0.05, rc = 5.

    python tests/golden/gen_golden.py --ref <reference checkout>
"""
import argparse
import importlib.util
import json
import os
import re
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def parse_cg(ref):
    src = open(os.path.join(ref, "include", "cg_coefficients_l3.cuh")).read()

    def arr(name):
        m = re.search(name + r"\[[^\]]*\](?:\[[^\]]*\])?\s*=\s*\{(.*?)\};", src, re.S)
        return [float(x) for x in re.findall(r"-?\d+\.?\d*(?:[eE]-?\d+)?", m.group(1))]

    bi = np.array(arr("BLOCK_INFO"), dtype=np.int64).reshape(34, 6)
    br = np.array(arr("BLOCK_RANGES"), dtype=np.int64).reshape(34, 2)
    ei = np.array(arr("ENTRY_INFO"), dtype=np.int64).reshape(611, 3)
    cf = np.array(arr("CG_COEFFS"), dtype=np.float64)
    assert cf.size == 611
    return {"source": "include/cg_coefficients_l3.cuh", "block_info": bi.tolist(), "block_ranges": br.tolist(),
            "entry_info": ei.tolist(), "coeffs": [float(np.float32(c)) for c in cf]}


def ref_autograd(ref):
    sys.modules.setdefault("_batmobile", types.ModuleType("_batmobile"))
    spec = importlib.util.spec_from_file_location("ref_autograd", os.path.join(ref, "python", "batmobile",
                                                                              "autograd.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sh_fixture(ref):
    m = ref_autograd(ref)
    g = torch.Generator().manual_seed(42)
    v = torch.randn(256, 3, generator=g, dtype=torch.float64)
    v = v / v.norm(dim=1, keepdim=True)
    s2, s3, eps = 1 / np.sqrt(2), 1 / np.sqrt(3), 1e-7
    special = torch.tensor([[1, 0, 0], [-1, 0, 0], [0, 1, 0], [0, -1, 0], [0, 0, 1], [0, 0, -1],
                            [s2, s2, 0], [s2, 0, s2], [0, s2, s2], [s3, s3, s3], [-s3, s3, s3],
                            [eps, 0, 1], [0, eps, 1], [eps, eps, 1], [eps, 0, -1]], dtype=torch.float64)
    special = special / special.norm(dim=1, keepdim=True)
    vec = torch.cat([v, special]).to(torch.float32)
    out = {"vectors": vec.numpy()}
    for L in range(5):
        out["Y%d" % L] = m._spherical_harmonics_forward_pytorch(vec.double(), L).numpy()
    gY = torch.randn(vec.shape[0], 16, generator=g, dtype=torch.float64)
    out["gY3"] = gY.numpy()
    out["gv3"] = m._spherical_harmonics_backward(vec.double(), gY, 3).numpy()
    return out


def nl_fixture():
    sys.path.insert(0, ROOT)
    from oracle import _native
    out = {}
    for n in (100, 300):
        box = float(np.float32(np.cbrt(np.float32(n) / np.float32(0.05))))
        pos = _native.ref_positions(n, box)
        ei, vec = _native.ref_brute_force(pos, box, 5.0)
        out["pos%d" % n] = pos.numpy()
        out["box%d" % n] = np.float32(box)
        out["ei%d" % n] = ei.numpy().astype(np.int32)
        out["vec%d" % n] = vec.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BATMOBILE_REF"))
    a = ap.parse_args()
    if not a.ref:
        ap.error("give --ref <reference checkout> or set BATMOBILE_REF")
    with open(os.path.join(HERE, "cg_l3.json"), "w") as f:
        json.dump(parse_cg(a.ref), f)
    np.savez_compressed(os.path.join(HERE, "sh_ref.npz"), **sh_fixture(a.ref))
    np.savez_compressed(os.path.join(HERE, "nl_ref.npz"), **nl_fixture())
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
