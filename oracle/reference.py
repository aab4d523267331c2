"""The reference's own Python package, for the tests (TEST INFRASTRUCTURE: tests/ only).

``oracle/build_ref.py`` copies nanocompile's package into the git-ignored ``oracle/_ref/py`` where
the checkout exists; the copy travels with the repository snapshot, so the tests that drive the
CUDA backend through the reference's ``Qwen2`` / ``Runner`` API import it on machines without the
checkout. Nothing here reads the checkout itself.
"""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent / "_ref" / "py"


def available() -> bool:
    return (PACKAGE / "nanocompile" / "__init__.py").exists()


def import_reference():
    """The ``nanocompile`` package from ``oracle/_ref/py``; raises ImportError when it was not built."""
    if not available():
        raise ImportError(f"{PACKAGE} holds no copy of the reference's nanocompile package: run "
                          f"`python oracle/build_ref.py` where the checkout is")
    os.environ.setdefault("NANOCOMPILE_CACHE", tempfile.mkdtemp(prefix="nanocompile-cache-"))
    sys.dont_write_bytecode = True
    if str(PACKAGE) not in sys.path:
        sys.path.insert(0, str(PACKAGE))
    import nanocompile

    loaded = Path(nanocompile.__file__).resolve()
    if PACKAGE not in loaded.parents:
        raise ImportError(f"nanocompile was already imported from {loaded}, not from {PACKAGE}")
    return nanocompile
