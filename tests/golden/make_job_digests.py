"""Writes tests/golden/job_digests.json: wc_job_digest of jobs built from
seeded roots across depths 1-4 (belief-heavy roots at depth 4, where the
builder's draw-transition and leaf-run reuse does the most), to pin the
builder's output byte for byte. Run from the repository root after a
deliberate change of the job format:

    python tests/golden/make_job_digests.py
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "war-chest-bot-9000-_b200"))

CASES = ([{"kind": "root", "seed": s, "plies": pl, "depth": d} for d in (1, 2, 3) for s in range(4) for pl in (20, 60)]
         + [{"kind": "wide", "seed": s, "ncfg": 256, "depth": 4} for s in (0, 5, 6, 7)])


def digests(wc):
    """The bench's cap-marker value (0.0) while building; the engine default
    (0.15, state.rs:27) restored after."""
    wc.set_cap_marker_value(0.0)
    out = []
    try:
        for c in CASES:
            cfg = wc.Cfg(depth=c["depth"], iters=8 if c["depth"] < 4 else 1024, snapshots=True, cfr=wc.Cfr.PLUS,
                         node_cap=200000)
            root = (wc.generate_root(c["seed"], c["plies"]) if c["kind"] == "root"
                    else wc.generate_wide_root(c["seed"], c["ncfg"]))
            out.append(dict(c, digest=str(wc.PackedJob.from_root(root, cfg).digest)))
    finally:
        wc.set_cap_marker_value(0.15)
    return out


if __name__ == "__main__":
    import warchest_b200 as wc

    path = os.path.join(ROOT, "tests", "golden", "job_digests.json")
    with open(path, "w") as f:
        json.dump(digests(wc), f, indent=1)
    print("wrote", path)
