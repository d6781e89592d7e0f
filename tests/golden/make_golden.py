"""Generate the golden fixtures for the slot allocator and the expert fetch.

Runs the REFERENCE's own Triton kernels -- ``_resolve_slots`` and
``_fetch_experts`` from ``bin/devcache.py`` -- on CPU tensors under
``TRITON_INTERPRET=1`` and records their outputs.  This needs the reference
checkout (``--reference``, or the ``D3_REFERENCE_DIR`` environment variable)
and only runs where that checkout exists; the committed ``.npz`` files travel
instead.

    python tests/golden/make_golden.py --reference <path-to-drama3-offloading>

Cases (each is a sequence of calls on one layer's tables, starting from
``init_dev_cache`` state, bin/devcache.py:138-167):

* small_dups      E=16  C=4   k=4   random ids WITH duplicates inside a call
* k_gt_c          E=16  C=3   k=8   more ids than slots (the reference's own
                                     hazard: a slot promised this call is reused)
* randperm_c16/32/64  E=64  k=8     torch.randperm ids, 40 calls, the capacities
                                     bin/test_devcache.py:47-76 uses
* zipf_c51        E=256 C=51  k=8   200 steps of the synthetic Zipf(1.1) trace,
                                     2048 slots / 40 layers (per-layer mode)
* zipf_c68        E=256 C=68  k=8   8 GiB cache per layer (68 slots)
* global_pool     E=10240 C=2048 k=8  keys layer*256+expert of the trace over
                                     one 2048-slot pool (global-pool mode)
* fetch           the byte copy of _fetch_experts, including a job count that
                  is smaller than the number of queued jobs
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    ap.add_argument("--out", default=str(HERE / "resolve_golden.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path-to-drama3-offloading> (or set D3_REFERENCE_DIR)")
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(args.reference) / "bin"))
    import torch
    import devcache  # the reference module
    from drama3_offloading_b200.trace import zipf_trace

    def run_case(E: int, C: int, calls: list[np.ndarray]) -> dict:
        slot_of = torch.full((E,), -1, dtype=torch.int32)
        slot_expert = torch.full((C,), -1, dtype=torch.int32)
        stamp = -torch.arange(C, 0, -1, dtype=torch.int64)
        step = torch.zeros(1, dtype=torch.int64)
        K = len(calls[0])
        out = torch.zeros(K, dtype=torch.int32)
        fs = torch.zeros(K, dtype=torch.int32)
        fe = torch.zeros(K, dtype=torch.int32)
        nm = torch.zeros(1, dtype=torch.int32)
        rec = {"out": [], "fslot": [], "fexp": [], "nmiss": []}
        for ids in calls:
            fs.fill_(-7)
            fe.fill_(-7)
            t = torch.from_numpy(np.asarray(ids, np.int32))
            devcache._resolve_slots[(1,)](t, slot_of, slot_expert, stamp, out, fs, fe, nm, step,
                                          K=K, C=C, num_warps=1)
            n = int(nm[0])
            rec["out"].append(out.numpy().copy())
            # entries past nmiss are not part of the contract; record -1 there
            f1 = fs.numpy().copy(); f1[n:] = -1
            f2 = fe.numpy().copy(); f2[n:] = -1
            rec["fslot"].append(f1)
            rec["fexp"].append(f2)
            rec["nmiss"].append(n)
        return {
            "E": np.int64(E), "C": np.int64(C), "ids": np.stack(calls).astype(np.int32),
            "out": np.stack(rec["out"]), "fslot": np.stack(rec["fslot"]),
            "fexp": np.stack(rec["fexp"]), "nmiss": np.asarray(rec["nmiss"], np.int32),
            "final_slot_of": slot_of.numpy().copy(),
            "final_slot_expert": slot_expert.numpy().copy(),
            "final_stamp": stamp.numpy().copy(), "final_step": step.numpy().copy(),
        }

    cases = {}
    rng = np.random.default_rng(1234)
    cases["small_dups"] = run_case(16, 4, [rng.integers(0, 16, 4) for _ in range(30)])
    cases["k_gt_c"] = run_case(16, 3, [rng.permutation(16)[:8] for _ in range(12)])
    torch.manual_seed(0)
    rp = [torch.randperm(64)[:8].numpy() for _ in range(40)]
    for c in (16, 32, 64):
        cases[f"randperm_c{c}"] = run_case(64, c, rp)
    tr = zipf_trace(steps=200, layers=40)
    cases["zipf_c51"] = run_case(256, 51, [tr[s, 0] for s in range(200)])
    cases["zipf_c68"] = run_case(256, 68, [tr[s, 1] for s in range(200)])
    gp = [(tr[s, l].astype(np.int64) + 256 * l).astype(np.int32)
          for s in range(3) for l in range(40)]
    cases["global_pool"] = run_case(10240, 2048, gp)

    flat = {}
    for name, d in cases.items():
        for key, v in d.items():
            flat[f"{name}/{key}"] = v

    # ---- fetch: the reference's _fetch_experts byte copy
    E, C, ELEMS, BLOCK = 12, 6, 384, 128
    host = torch.from_numpy(rng.integers(0, 256, (E, ELEMS), dtype=np.uint8))
    cache = torch.full((C, ELEMS), 0xA5, dtype=torch.uint8)
    fslot = torch.tensor([4, 0, 5, 2, 1, 3], dtype=torch.int32)
    fexp = torch.tensor([7, 11, 0, 3, 9, 5], dtype=torch.int32)
    nmiss = torch.tensor([4], dtype=torch.int32)   # fewer jobs than queued entries
    K = 6
    grid = (K * ((ELEMS + BLOCK - 1) // BLOCK),)
    devcache._fetch_experts[grid](host.reshape(-1), cache.reshape(-1), fslot, fexp, nmiss,
                                  ELEMS=ELEMS, BLOCK=BLOCK, num_warps=4)
    flat.update({"fetch/host": host.numpy(), "fetch/cache_after": cache.numpy(),
                 "fetch/fslot": fslot.numpy(), "fetch/fexp": fexp.numpy(),
                 "fetch/nmiss": nmiss.numpy(), "fetch/fill": np.uint8(0xA5)})
    np.savez_compressed(args.out, **flat)
    print(f"wrote {args.out}: {len(cases)} resolve cases + fetch")
    for name, d in cases.items():
        print(f"  {name:14s} E={int(d['E']):5d} C={int(d['C']):4d} calls={len(d['ids']):3d} "
              f"misses={int(d['nmiss'].sum())}")


if __name__ == "__main__":
    main()
