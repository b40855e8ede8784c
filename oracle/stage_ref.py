"""Stage the reference's operator sources for the GPU-side reference runs.

TEST INFRASTRUCTURE ONLY.  The reference (qhfan/FlashPrefill) is Python + Triton; its operator
is the package ``ops/`` (``ops/__init__.py``, ``ops/flashprefill_native_forward.py``,
``ops/flashprefill_varlen_func.py``).  Its checkout is not present on the GPU hosts, so this
recipe copies those three files byte for byte, unmodified, into ``oracle/_ref/ops/``.  That
folder is git-ignored (the reference's sources are never committed here) and travels with the
working tree like the built library.  Only the reference-side checks (``oracle/triton_ref.py``:
the GPU parity tests against the reference and bench.py's Triton baseline leg) load it.

    python oracle/stage_ref.py [--ref <reference checkout>]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref", "ops")
FILES = ("__init__.py", "flashprefill_native_forward.py", "flashprefill_varlen_func.py")
DEFAULT_REF = os.environ.get("FLASHPREFILL_REFERENCE", "/root/reference")


def stage(ref: str = DEFAULT_REF) -> str | None:
    """Copy the reference's ops/ files into oracle/_ref/ops/; returns the folder, or None when
    no reference checkout is available (the staged copy, if any, is then left as it is)."""
    src = os.path.join(ref, "ops")
    if not all(os.path.isfile(os.path.join(src, f)) for f in FILES):
        return None
    os.makedirs(DEST, exist_ok=True)
    lines = []
    for f in FILES:
        shutil.copyfile(os.path.join(src, f), os.path.join(DEST, f))
        lines.append(f"{hashlib.sha256(open(os.path.join(DEST, f), 'rb').read()).hexdigest()}  ops/{f}")
    with open(os.path.join(os.path.dirname(DEST), "SHA256SUMS"), "w") as fh:
        fh.write("\n".join(lines) + "\n")
    return DEST


def staged() -> bool:
    return all(os.path.isfile(os.path.join(DEST, f)) for f in FILES)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=DEFAULT_REF)
    d = stage(ap.parse_args().ref)
    print(d if d else "reference checkout not found; nothing staged")
