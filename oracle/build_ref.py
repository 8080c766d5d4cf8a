"""Compile the reference package for the timed CPU baseline (bench infrastructure only).

    python oracle/build_ref.py [--reference DIR]      (default: $ECOINT8_REFERENCE)

The reference (eco-int8-opt 0.4.9) is pure Python on PyTorch.  This recipe
byte-compiles its ``ecoint8`` package where it lies into sourceless bytecode, one
compiled module per source module, stored in the archive ``oracle/_ref/ecoint8.zip``
(importable without the sources through Python's zip importer; the GPU machines run
the same Python version).  No source file is copied.
``bench.py`` imports the package from there to time the reference's own strict
step on the host cores: the ``--impl reference`` arm and ``cpu_baseline``.
``oracle/_ref`` is listed in ``.gitignore`` and is never committed.
"""

from __future__ import annotations

import argparse
import importlib.util
import marshal
import os
import pathlib
import sys
import zipfile

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
ARCHIVE = OUT / "ecoint8.zip"


def build(reference: str | os.PathLike | None = None) -> pathlib.Path | None:
    """Compile ``<reference>/ecoint8`` into ``oracle/_ref``; None when no reference is given."""
    ref = reference or os.environ.get("ECOINT8_REFERENCE")
    if not ref:
        return None
    pkg = pathlib.Path(ref) / "ecoint8"
    if not (pkg / "__init__.py").exists():
        raise FileNotFoundError(f"no ecoint8 package under {ref}")
    OUT.mkdir(exist_ok=True)
    tmp = ARCHIVE.with_suffix(".tmp")
    with zipfile.ZipFile(tmp, "w", zipfile.ZIP_DEFLATED) as z:
        for src in sorted(pkg.rglob("*.py")):
            rel = src.relative_to(pkg)
            code = compile(src.read_bytes(), f"ecoint8/{rel}", "exec", dont_inherit=True)
            # a sourceless .pyc: magic, flags 0 (timestamp-based), mtime, size, marshalled code
            head = importlib.util.MAGIC_NUMBER + (0).to_bytes(4, "little") + (0).to_bytes(4, "little") \
                + (0).to_bytes(4, "little")
            z.writestr(str(pathlib.PurePosixPath("ecoint8", rel.with_suffix(".pyc"))), head + marshal.dumps(code))
    os.replace(tmp, ARCHIVE)
    (OUT / "BUILT_FROM").write_text(f"{pkg.resolve()}\npython {sys.version.split()[0]}\n")
    return ARCHIVE


def load():
    """Import the compiled reference (``ecoint8`` of oracle/_ref) for CPU timing, or None.

    Triton is hidden from it: the strict path never uses it, and its JIT decorators
    need the sources that the bytecode build does not carry (the reference then takes
    its own CPU-install branch, ``TRITON_AVAILABLE = False``).
    """
    if not ARCHIVE.exists():
        return None
    if "ecoint8" in sys.modules and not getattr(sys.modules["ecoint8"], "__file__", "").startswith(str(OUT)):
        raise RuntimeError("another ecoint8 package is already imported in this process")
    sys.modules.setdefault("triton", None)
    sys.path.insert(0, str(ARCHIVE))
    try:
        import ecoint8  # noqa: F401
        import ecoint8.strict as strict
        import ecoint8.quant as quant
    finally:
        sys.path.remove(str(ARCHIVE))
    assert ecoint8.__file__.startswith(str(ARCHIVE))
    return {"ecoint8": ecoint8, "strict": strict, "quant": quant, "version": ecoint8.__version__}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (default: $ECOINT8_REFERENCE)")
    a = ap.parse_args()
    out = build(a.reference)
    if out is None:
        raise SystemExit("give --reference or set ECOINT8_REFERENCE")
    print(out)
