"""Derive one residual direction from captured development probes (the reference's
`tools/weight-space/derive_direction.py` role).

    python -m dllm_qwen38_b200.weight_space.derive_direction --capture CAP_DIR --output OUT_DIR
           --layer L --prompts 8 --pairs 0:1 2:3 4:5 --reset 6:7 --min-mean-cosine 0.3

Each pair (early, late) contributes the difference of the final residuals late - early at layer L;
the reset pair are two prompts with an identical prefix whose residuals must agree (max |diff|
<= 1e-5: a control that the capture is deterministic). Pairs and the reset pair must cover every
prompt exactly once. The unit differences' mean pairwise cosine must reach the gate; if it does,
the normalised mean of the unit differences is saved as OUT_DIR/direction-L.npy. OUT_DIR must be
new; derivation.json records norms, cosines, the gate and every input file's digest.
"""

from __future__ import annotations

import argparse
import json
import pathlib

import numpy as np

from .capture_data import load_vectors
from .common import digest

RESET_TOL = 1e-5


def derive(capture, output, layer: int, prompts: int, pairs, reset, minimum: float) -> dict:
    if not np.isfinite(minimum) or not -1.0 <= minimum <= 1.0:
        raise ValueError("the cosine gate must lie in [-1, 1]")
    idx = [i for p in pairs for i in p] + list(reset)
    if len(pairs) < 2 or any(len(p) != 2 for p in pairs) or len(reset) != 2:
        raise ValueError("need at least two (early, late) pairs and one reset pair")
    if len(set(idx)) != len(idx) or set(idx) != set(range(prompts)):
        raise ValueError("pairs and the reset pair must cover every prompt exactly once")
    vecs, acct = load_vectors(capture, prompts, [layer])
    reset_delta = float(np.max(np.abs(vecs[(reset[0], layer)] - vecs[(reset[1], layer)])))
    if reset_delta > RESET_TOL:
        raise ValueError("identical-prefix reset control failed")
    diffs = [vecs[(late, layer)].astype(np.float64) - vecs[(early, layer)] for early, late in pairs]
    norms = [float(np.linalg.norm(v)) for v in diffs]
    if not np.isfinite(norms).all() or min(norms) <= 1e-8:
        raise ValueError("a pair shows no contrast")
    units = [v / n for v, n in zip(diffs, norms)]
    cos = [float(units[i] @ units[j]) for i in range(len(units)) for j in range(i + 1, len(units))]
    mean_cos = float(np.mean(cos))
    direction = np.mean(units, axis=0)
    dn = float(np.linalg.norm(direction))
    if not np.isfinite(dn) or dn <= 1e-8:
        raise ValueError("the mean direction vanished")
    direction = (direction / dn).astype(np.float32)
    out = pathlib.Path(output)
    out.mkdir()  # a changed declaration needs a fresh directory
    rep = {"layer": layer, "pairs": [list(p) for p in pairs], "reset_pair": list(reset),
           "minimum_mean_pair_cosine": minimum, "pair_delta_norms": norms, "pair_cosines": cos,
           "mean_pair_cosine": mean_cos, "reset_control_max_abs": reset_delta, "accounting": acct,
           "source_sha256": digest(__file__),
           "capture_file_sha256": {p.name: digest(p) for p in sorted(pathlib.Path(capture).iterdir()) if p.is_file()},
           "gate_passed": mean_cos >= minimum,
           "qualification": "an association on saved development prompts; not evidence of a causal mechanism"}
    if rep["gate_passed"]:
        target = out / f"direction-{layer}.npy"
        np.save(target, direction)
        rep["direction_sha256"] = digest(target)
    (out / "derivation.json").write_text(json.dumps(rep, indent=2) + "\n")
    return rep


def _pair(v: str):
    t = tuple(int(x) for x in v.split(":"))
    if len(t) != 2:
        raise argparse.ArgumentTypeError("use early:late prompt indexes")
    return t


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--capture", required=True, type=pathlib.Path)
    p.add_argument("--output", required=True, type=pathlib.Path)
    p.add_argument("--layer", required=True, type=int)
    p.add_argument("--prompts", type=int, default=8)
    p.add_argument("--pairs", nargs="+", required=True, type=_pair)
    p.add_argument("--reset", required=True, type=_pair)
    p.add_argument("--min-mean-cosine", required=True, type=float)
    a = p.parse_args(argv)
    r = derive(a.capture, a.output, a.layer, a.prompts, a.pairs, a.reset, a.min_mean_cosine)
    print(json.dumps({k: r[k] for k in ("layer", "gate_passed", "mean_pair_cosine", "reset_control_max_abs")},
                     indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
