"""Install the unmodified tensorshrink reference into `baseline/_ref/` for
`bench.py --impl reference`.

The reference checkout has neither `setup.py` nor `pyproject.toml`, so
`pip install --target baseline/_ref <checkout>` stops with "not
installable". This recipe does what that install would: it places the
checkout's Python files, unchanged, as the package `tensorshrink` under
`baseline/_ref/` (git-ignored; it travels with the working tree to the GPU
host). Nothing is edited.

The package's `__init__` imports `container.py`, which needs the
`zstandard` module, absent from this image; `bench.py` therefore imports
`tensorshrink.codec` and `tensorshrink.modules` as submodules of a bare
package object (the hot path lives entirely in those two files plus
`triton_kernels.py`).

Usage: python baseline/install_ref.py [REFERENCE_CHECKOUT]
"""

from __future__ import annotations

import shutil
import sys
from pathlib import Path

DEST = Path(__file__).resolve().parent / "_ref" / "tensorshrink"


def main() -> int:
    if len(sys.argv) < 2:
        print("usage: python baseline/install_ref.py REFERENCE_CHECKOUT", file=sys.stderr)
        return 2
    src = Path(sys.argv[1])
    files = sorted(src.glob("*.py"))
    if not (src / "modules.py").exists() or not files:
        print(f"{src} does not look like the tensorshrink checkout", file=sys.stderr)
        return 1
    DEST.mkdir(parents=True, exist_ok=True)
    for f in files:
        shutil.copyfile(f, DEST / f.name)
    lic = src / "LICENSE"
    if lic.exists():
        shutil.copyfile(lic, DEST / "LICENSE")
    print(f"installed {len(files)} files into {DEST}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
