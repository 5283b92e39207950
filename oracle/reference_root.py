"""Where the reference project's source tree is, if it is present at all.

Test infrastructure only.  Resolved from the LAZY_RECALL_REFERENCE
environment variable, else from the "reference_path" field of the
repository's BASELINE.json (the build environment's record of where the
reference is mounted).  Returns None when neither names an existing tree: the
checkers built from the reference (oracle/_ref) are then used as already
built, and the recipes that need the sources skip or refuse.
"""
from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Optional

ROOT = Path(__file__).resolve().parent.parent


def reference_root() -> Optional[Path]:
    named = os.environ.get("LAZY_RECALL_REFERENCE")
    if not named:
        record = ROOT / "BASELINE.json"
        if record.exists():
            try:
                named = json.loads(record.read_text()).get("reference_path")
            except (OSError, ValueError):
                named = None
    if not named:
        return None
    root = Path(named)
    return root if (root / "csrc" / "scoring.cu").exists() else None
