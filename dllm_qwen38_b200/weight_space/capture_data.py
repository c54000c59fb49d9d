"""Read the output directory of this framework's `capture` tool (native_tools/capture.cpp) into
final-position residual vectors, with the run's accounting checked first (the reference's
`tools/weight-space/capture_data.py:8-37` role, for our capture format):

  DIR/status.json   {"ok", "prompts", "tensors", "layer_visits", "error"}
  DIR/index.jsonl   {"prompt", "layer", "file", "rows", "cols", "bytes"} per tensor
  DIR/<file>        float32 little-endian [rows, cols]

load_vectors(dir, prompts, layers) -> ({(prompt, layer): float32 [cols]}, accounting): the last
row of each [T, D] residual (the final prompt position). The status must be ok, every prompt must
have one tensor per requested layer, byte counts must match the shapes, and values must be finite.
"""

from __future__ import annotations

import json
import pathlib

import numpy as np


def load_vectors(directory, prompts: int, layers, width: int | None = None):
    d = pathlib.Path(directory)
    st = json.loads((d / "status.json").read_text())
    want = {(p, int(layer)) for p in range(prompts) for layer in layers}
    if not st.get("ok") or st.get("prompts") != prompts or st.get("error"):
        raise ValueError("capture run did not complete")
    rows = [json.loads(x) for x in (d / "index.jsonl").read_text().splitlines() if x.strip()]
    if len(rows) != st.get("tensors") or len(rows) != len(want):
        raise ValueError("capture tensor accounting failed")
    out = {}
    for r in rows:
        key = (int(r["prompt"]), int(r["layer"]))
        if key not in want or key in out:
            raise ValueError(f"unexpected or repeated tensor {key}")
        n, w = int(r["rows"]), int(r["cols"])
        if width is not None and w != width:
            raise ValueError(f"residual width {w}, expected {width}")
        vals = np.fromfile(d / r["file"], dtype="<f4")
        if vals.nbytes != int(r["bytes"]) or vals.size != n * w or n < 1:
            raise ValueError(f"byte count mismatch for {r['file']}")
        if not np.isfinite(vals).all():
            raise ValueError(f"non-finite residual in {r['file']}")
        out[key] = vals.reshape(n, w)[-1].copy()
    if set(out) != want:
        raise ValueError("missing residuals")
    return out, {"capture_status": st, "vectors": len(out)}
