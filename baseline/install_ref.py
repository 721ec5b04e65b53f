"""Install the unmodified reference build under ``baseline/_ref``.

    python baseline/install_ref.py [--source PATH] [--force]

First tries the offline pip install the benchmark protocol prescribes
(``pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
--target baseline/_ref <source>``).  The reference tree carries no packaging
metadata (neither ``setup.py`` nor ``pyproject.toml``), so pip refuses it; the
script then copies the tree verbatim and checks every copied file against its
source by SHA-256.  Nothing in the copy is edited, added or removed: the
reference arm of ``bench.py`` imports it as it is.  The reference's own JIT
build of its event bridge writes under ``/tmp``, never into the copy.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
from pathlib import Path
import shutil
import subprocess
import sys

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"
DEFAULT_SOURCE = "/root/reference"


def _digest_tree(root: Path) -> dict[str, str]:
    out = {}
    for path in sorted(root.rglob("*")):
        if path.is_file() and "__pycache__" not in path.parts:
            out[str(path.relative_to(root))] = hashlib.sha256(path.read_bytes()).hexdigest()
    return out


def _pip_install(source: str, target: Path) -> tuple[bool, str]:
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--find-links", "/opt/wheelhouse", "--target", str(target), source]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    tail = (proc.stdout + proc.stderr).strip().splitlines()[-1:] or [""]
    return proc.returncode == 0, tail[0]


def install(source: str = DEFAULT_SOURCE, force: bool = False) -> dict:
    src = Path(source)
    if not (src / "scripts" / "run_r4_a0_c0_full_moe.py").exists():
        return {"ok": False, "how": "none", "why": f"no reference tree at {source}"}
    if TARGET.exists():
        if not force and _digest_tree(TARGET) == _digest_tree(src):
            return {"ok": True, "how": "present", "files": len(_digest_tree(TARGET))}
        shutil.rmtree(TARGET)
    ok, msg = _pip_install(source, TARGET)
    if ok:
        return {"ok": True, "how": "pip", "detail": msg}
    if TARGET.exists():
        shutil.rmtree(TARGET)
    shutil.copytree(src, TARGET, symlinks=True, ignore=shutil.ignore_patterns("__pycache__"))
    want, got = _digest_tree(src), _digest_tree(TARGET)
    if want != got:
        shutil.rmtree(TARGET)
        return {"ok": False, "how": "copy", "why": "copied tree differs from the source"}
    return {"ok": True, "how": "verbatim copy", "pip": msg, "files": len(got)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--source", default=os.environ.get("RAICCL_REFERENCE_SOURCE", DEFAULT_SOURCE))
    ap.add_argument("--force", action="store_true", help="reinstall even if an identical copy is present")
    args = ap.parse_args()
    rec = install(args.source, args.force)
    print(json.dumps(rec))
    raise SystemExit(0 if rec["ok"] else 1)


if __name__ == "__main__":
    main()
