"""Exclusive ownership receipt for a controller's output directory (the reference's
`tools/weight-space/controller_claim.py:10-21` role): `claim(dir, protocol_sha256)` creates
`controller-owner.json` with O_CREAT | O_EXCL, so two controllers can never both believe they own
the directory; the receipt stays after completion, so a rerun needs a fresh directory."""

from __future__ import annotations

import datetime
import json
import os
import pathlib
import re
import sys


def claim(directory, protocol_sha256: str) -> dict:
    root = pathlib.Path(directory).resolve(strict=True)
    if not root.is_dir():
        raise ValueError("an existing output directory is required")
    if not re.fullmatch(r"[0-9a-f]{64}", protocol_sha256 or ""):
        raise ValueError("a lowercase hex SHA-256 of the protocol is required")
    receipt = {"pid": os.getpid(), "protocol_sha256": protocol_sha256, "argv": list(sys.argv),
               "started_utc": datetime.datetime.now(datetime.timezone.utc).isoformat()}
    fd = os.open(root / "controller-owner.json", os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o600)
    with os.fdopen(fd, "w") as f:
        json.dump(receipt, f, indent=2)
        f.write("\n")
    return receipt
