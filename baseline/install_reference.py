"""Install the unmodified reference tree under baseline/_ref for the reference GPU timings.

The stock command is tried first:

    python -m pip install --no-index --no-build-isolation \
        --find-links /opt/wheelhouse --target baseline/_ref <reference root>

The reference ships no setup.py / pyproject.toml, so pip refuses it.  Its
Python code then goes into baseline/_ref the way its own scripts import it
(``sys.path`` holding the tree's root and ``src/``): the packages
``kernels`` (the Triton kernels, kernels/diffusion_triton.py), ``cta``
(src/cta: the vLLM post-attention mixer and the PyTorch stencil) and
``models`` (src/models: the PDE layers), copied file for file and unchanged.
INSTALL.json records the pip outcome and the sha256 of every copied file.

baseline/_ref is ignored by git: the reference is run beside this package,
never shipped in it.  Usage: ``python baseline/install_reference.py --ref
<reference root>`` (or CTA_REFERENCE_ROOT in the environment).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"
# (source inside the reference tree, destination package under baseline/_ref)
PACKAGES = [("kernels", "kernels"), ("src/cta", "cta"), ("src/models", "models")]


def _sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def install(ref: Path) -> dict:
    ref = ref.resolve()
    if not (ref / "kernels" / "diffusion_triton.py").is_file():
        raise SystemExit(f"{ref} does not hold kernels/diffusion_triton.py")
    TARGET.mkdir(parents=True, exist_ok=True)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           "/opt/wheelhouse", "--target", str(TARGET), str(ref)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    pip_msg = (res.stderr.strip().splitlines() or [""])[-1] if res.returncode else "installed"
    record = {"source": str(ref), "pip_returncode": res.returncode, "pip_result": pip_msg, "files": {}}
    if res.returncode != 0:
        for src, dst in PACKAGES:
            s, d = ref / src, TARGET / dst
            if d.exists():
                shutil.rmtree(d)
            shutil.copytree(s, d, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
            for f in sorted(d.rglob("*")):
                if f.is_file():
                    record["files"][str(f.relative_to(TARGET))] = _sha256(f)
        # the copied files must equal the reference's byte for byte
        for rel, digest in record["files"].items():
            top, rest = rel.split("/", 1)
            src = dict((b, a) for a, b in PACKAGES)[top]
            assert _sha256(ref / src / rest) == digest, rel
    (TARGET / "INSTALL.json").write_text(json.dumps(record, indent=1))
    return record


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ref", default=os.environ.get("CTA_REFERENCE_ROOT"),
                    help="root of the reference tree (or CTA_REFERENCE_ROOT)")
    args = ap.parse_args(argv)
    if not args.ref:
        ap.error("give --ref or set CTA_REFERENCE_ROOT")
    rec = install(Path(args.ref))
    print(json.dumps({"pip": rec["pip_result"], "files": len(rec["files"])}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
