"""Generate the golden vectors by running the REFERENCE optimizer on the CPU.

Run once, in a container where the reference checkout exists:

    python tests/golden/make_golden.py --ref <reference checkout> [case ...]

(or set SMO_REFERENCE_DIR instead of passing --ref).

For every case of cases.py it builds the seeded synthetic params, runs the
reference's own ``SMO8bit`` / ``SMO`` (smo/optimizers/spatial_8bit.py,
smo/optimizers/spatial.py) for the case's steps with the seeded synthetic
grads, and writes ``<case>.npz`` next to this script: the final optimizer
state arrays, the state metadata, and the final params (a strided sample for
the large single-weight case).  For the cases in STATE_DICT_CASES it also
writes ``<case>.state.pt``: the reference optimizer's own ``state_dict()``,
saved with ``torch.save``, which the tests load into the drop-in optimizer.
The tests compare the CPU oracle and the CUDA library against these files;
nothing at test time imports the reference.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# cases whose final reference state_dict() is saved as written by the reference
STATE_DICT_CASES = ("s8_groups", "s8_128x256_band_wd", "smo_groups")
ROOT = os.path.dirname(os.path.dirname(HERE))


def main():
    ap = argparse.ArgumentParser()
    env_ref = os.environ.get("SMO_REFERENCE_DIR")
    ap.add_argument("--ref", default=env_ref, required=env_ref is None,
                    help="checkout of the reference (the directory holding the smo package)")
    ap.add_argument("cases", nargs="*")
    args = ap.parse_args()

    sys.path.insert(0, ROOT)
    sys.path.insert(0, args.ref)
    import torch
    from smo.optimizers.spatial import SMO
    from smo.optimizers.spatial_8bit import SMO8bit

    sys.path.insert(0, HERE)
    import cases as C

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    names = args.cases or list(C.CASES)
    for name in names:
        case = C.CASES[name]
        tdtype = getattr(torch, C.case_dtype(case))
        params = [torch.nn.Parameter(torch.from_numpy(a.copy()).to(tdtype)) for a in C.case_params(case)]
        groups = C.case_groups(case, params)
        cls = SMO8bit if case["opt"] == "SMO8bit" else SMO
        opt = cls(groups, **case["kwargs"])
        torch.manual_seed(case["seed"])  # permute_basis draws its permutations at the first step
        for step in range(1, case["steps"] + 1):
            for p, g in zip(params, C.case_grads(case, step)):
                p.grad = torch.from_numpy(g.copy()).to(tdtype)
            opt.step()
        out = {}
        meta = {"case": name, "torch": torch.__version__, "param_dtype": C.case_dtype(case), "tensors": []}
        stride = case.get("sample_stride")
        for i, p in enumerate(params):
            arr = p.detach().float().numpy().reshape(-1)  # half-precision values are exact in fp32
            if stride:
                out[f"{i}.param_sample"] = arr[C.sample_indices(arr.size, stride)].copy()
            else:
                out[f"{i}.param"] = arr.copy()
            st = opt.state[p]
            tmeta = {}
            for k in C.STATE_META_KEYS:
                if k in st:
                    v = st[k]
                    tmeta[k] = list(v) if isinstance(v, tuple) else v
            meta["tensors"].append(tmeta)
            for k in C.STATE_ARRAY_KEYS:
                if k in st:
                    t = st[k].detach()
                    out[f"{i}.{k}"] = (t.float() if t.is_floating_point() else t).numpy().copy()
        if name in STATE_DICT_CASES:
            sd_path = os.path.join(HERE, f"{name}.state.pt")
            torch.save(opt.state_dict(), sd_path)
            print(f"{name}: state_dict {os.path.getsize(sd_path) / 1024:.1f} KiB")
        out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"{name}: {os.path.getsize(path) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
