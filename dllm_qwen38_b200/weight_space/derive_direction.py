"""Derive one residual direction from captured development probes (the role of the reference's
`tools/weight-space/derive_direction.py:13-74`).

    python -m dllm_qwen38_b200.weight_space.derive_direction --capture CAP_DIR --output OUT_DIR
           --layer L --prompts 8 --pairs 0:1 2:3 4:5 --reset 6:7 --min-mean-cosine 0.3

The declaration names, for one layer, some (early, late) prompt pairs and one reset pair. The
reset pair are two prompts sharing an identical prefix; their captured residuals must agree to
1e-5, which shows that the capture is deterministic before any contrast is trusted. Every other
pair contributes its contrast late - early. The contrasts are normalised to unit rows of a matrix
U; their agreement is the mean of the off-diagonal upper triangle of the Gram matrix U U^T. When
that mean reaches the declared gate, the direction (the normalised mean of the rows of U) is
written to OUT_DIR/direction-L.npy. OUT_DIR must not exist yet: a changed declaration gets a
fresh directory. derivation.json records the statistics, the gate and the digest of every input.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import pathlib

import numpy as np

from .capture_data import load_vectors
from .common import digest

RESET_TOL = 1e-5
TINY = 1e-8
QUALIFICATION = "an association on saved development prompts; not evidence of a causal mechanism"


@dataclasses.dataclass(frozen=True)
class Declaration:
    layer: int
    prompts: int
    pairs: tuple
    reset: tuple
    gate: float

    def check(self) -> None:
        """Raise ValueError unless the declaration is usable: a gate in [-1, 1], at least two
        contrast pairs, and pairs plus reset pair partitioning the prompts."""
        if not (np.isfinite(self.gate) and abs(self.gate) <= 1.0):
            raise ValueError("the cosine gate must lie in [-1, 1]")
        if len(self.pairs) < 2 or len(self.reset) != 2 or any(len(p) != 2 for p in self.pairs):
            raise ValueError("need at least two (early, late) pairs and one reset pair")
        used = sorted([i for p in self.pairs for i in p] + list(self.reset))
        if used != list(range(self.prompts)):
            raise ValueError("pairs and the reset pair must cover every prompt exactly once")


def contrast_statistics(contrasts: np.ndarray) -> dict:
    """Statistics of a [pairs, dim] contrast matrix (float64): row norms, pairwise cosines of the
    unit rows (upper triangle of their Gram matrix, row-major), their mean, and the unit mean
    direction. Raises when a contrast or the mean direction is (numerically) zero."""
    norms = np.linalg.norm(contrasts, axis=1)
    if not np.all(np.isfinite(norms)) or norms.min() <= TINY:
        raise ValueError("a pair shows no contrast")
    unit = contrasts / norms[:, None]
    gram = unit @ unit.T
    iu = np.triu_indices(len(unit), k=1)
    mean_dir = unit.mean(axis=0)
    size = float(np.linalg.norm(mean_dir))
    if not np.isfinite(size) or size <= TINY:
        raise ValueError("the mean direction vanished")
    cos = gram[iu]
    return {"norms": norms.tolist(), "cosines": cos.tolist(), "mean_cosine": float(cos.mean()),
            "direction": (mean_dir / size).astype(np.float32)}


def derive(capture, output, layer: int, prompts: int, pairs, reset, minimum: float) -> dict:
    decl = Declaration(layer, prompts, tuple(tuple(p) for p in pairs), tuple(reset), minimum)
    decl.check()
    vecs, acct = load_vectors(capture, prompts, [layer])
    a, b = decl.reset
    reset_delta = float(np.abs(vecs[(a, layer)] - vecs[(b, layer)]).max())
    if reset_delta > RESET_TOL:
        raise ValueError("identical-prefix reset control failed")
    contrasts = np.stack([vecs[(late, layer)].astype(np.float64) - vecs[(early, layer)]
                          for early, late in decl.pairs])
    stats = contrast_statistics(contrasts)
    out = pathlib.Path(output)
    out.mkdir()  # refuses an existing directory
    passed = stats["mean_cosine"] >= decl.gate
    report = {
        "layer": layer, "pairs": [list(p) for p in decl.pairs], "reset_pair": list(decl.reset),
        "minimum_mean_pair_cosine": decl.gate, "pair_delta_norms": stats["norms"],
        "pair_cosines": stats["cosines"], "mean_pair_cosine": stats["mean_cosine"],
        "reset_control_max_abs": reset_delta, "accounting": acct, "source_sha256": digest(__file__),
        "capture_file_sha256": {f.name: digest(f) for f in sorted(pathlib.Path(capture).iterdir()) if f.is_file()},
        "gate_passed": passed, "qualification": QUALIFICATION,
    }
    if passed:
        path = out / f"direction-{layer}.npy"
        np.save(path, stats["direction"])
        report["direction_sha256"] = digest(path)
    (out / "derivation.json").write_text(json.dumps(report, indent=2) + "\n")
    return report


def _index_pair(text: str) -> tuple:
    parts = text.split(":")
    if len(parts) != 2 or not all(p.strip().lstrip("-").isdigit() for p in parts):
        raise argparse.ArgumentTypeError("use early:late prompt indexes")
    return int(parts[0]), int(parts[1])


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--capture", required=True, type=pathlib.Path)
    p.add_argument("--output", required=True, type=pathlib.Path)
    p.add_argument("--layer", required=True, type=int)
    p.add_argument("--prompts", type=int, default=8)
    p.add_argument("--pairs", nargs="+", required=True, type=_index_pair)
    p.add_argument("--reset", required=True, type=_index_pair)
    p.add_argument("--min-mean-cosine", required=True, type=float)
    a = p.parse_args(argv)
    rep = derive(a.capture, a.output, a.layer, a.prompts, a.pairs, a.reset, a.min_mean_cosine)
    summary = {"layer": rep["layer"], "gate_passed": rep["gate_passed"], "mean_pair_cosine": rep["mean_pair_cosine"],
               "reset_control_max_abs": rep["reset_control_max_abs"]}
    print(json.dumps(summary, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
