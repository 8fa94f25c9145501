"""Build the sm_100a shared library in place (reference: build_so.py:1-102,
which targets sm_80..sm_120 and has no sm_100 image)."""
from __future__ import annotations

import importlib.util
from pathlib import Path

_BUILD = Path(__file__).resolve().parent.parent / "build.py"


def build(force: bool = False) -> Path:
    """Compile libmosyne_bposit.so next to this package and return its path."""
    spec = importlib.util.spec_from_file_location("_mosyne_bposit_build", _BUILD)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=force)


def main() -> None:
    print(build())


if __name__ == "__main__":
    main()
