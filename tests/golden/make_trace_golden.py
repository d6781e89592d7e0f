"""Generate the real-trace fixture: the reference's captured decode routing
(``notes/route-trace-512.json``: 211 decode frames x 40 layers x top-8, the
trace behind the reference's published hit-rate table) as an int16 array,
with the hit counts of the reference's own cache simulator
(``bin/simulate_cache.py`` ``simulate``, per-layer LRU and LFU) at several
per-layer capacities.

    python tests/golden/make_trace_golden.py --reference <path-to-drama3-offloading>

(or set D3_REFERENCE_DIR).  Only runs where the reference checkout exists;
the committed ``route_trace_512.npz`` travels instead.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CAPS = (51, 68, 85, 113, 127, 170)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    ap.add_argument("--out", default=str(HERE / "route_trace_512.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path-to-drama3-offloading> (or set D3_REFERENCE_DIR)")
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "bin"))
    import simulate_cache  # the reference module (standard library only)

    data = json.loads((ref / "notes" / "route-trace-512.json").read_text())
    dec = [r for r in data["records"] if r["phase"] == "decode"]
    per_layer = [[] for _ in range(40)]
    for r in dec:
        ids = r["ids"][0] if isinstance(r["ids"][0], list) else r["ids"]
        per_layer[r["layer"]].append(ids)
    steps = min(len(x) for x in per_layer)
    trace = np.array([[per_layer[l][s] for l in range(40)] for s in range(steps)], np.int16)
    lru, lfu, total = [], [], []
    for cap in CAPS:
        h, t = simulate_cache.simulate(dec, cap, "lru")
        hf, tf = simulate_cache.simulate(dec, cap, "lfu")
        lru.append(h); lfu.append(hf); total.append(t)
    np.savez_compressed(args.out, trace=trace, caps=np.array(CAPS), ref_lru_hits=np.array(lru),
                        ref_lfu_hits=np.array(lfu), total=np.array(total))
    print(f"wrote {args.out}: trace {trace.shape}, lru {lru}, lfu {lfu}, total {total}")


if __name__ == "__main__":
    main()
