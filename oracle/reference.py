"""Test infrastructure only: import the compiled reference under its own module name.

oracle/build_ref.sh installs the unmodified reference package (luisrodolfo10/
diff_gabor_splatting v0.1.1, src/gabor_splatting/) into oracle/_ref/.  Its import name,
``gabor_splatting``, is also the name this repository's drop-in package answers to, so
the parity tests and the reference timing script load the reference as ``gs_reference``
instead: ``gs_reference.rasterize_gabors``, ``gs_reference.rendering``,
``gs_reference._C`` (its relative imports resolve inside that package).  Nothing in the
product imports this module.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent / "_ref" / "gabor_splatting"
NAME = "gs_reference"


def available() -> bool:
    return (REF_DIR / "__init__.py").exists() and any(REF_DIR.glob("_C*.so"))


def load():
    """The reference package (module ``gs_reference``); ImportError when not built."""
    if NAME in sys.modules:
        return sys.modules[NAME]
    if not available():
        raise ImportError("the compiled reference is not in oracle/_ref (oracle/build_ref.sh)")
    spec = importlib.util.spec_from_file_location(
        NAME, REF_DIR / "__init__.py", submodule_search_locations=[str(REF_DIR)])
    module = importlib.util.module_from_spec(spec)
    sys.modules[NAME] = module
    try:
        spec.loader.exec_module(module)
    except BaseException:
        del sys.modules[NAME]
        raise
    importlib.import_module(NAME + ".rendering")
    importlib.import_module(NAME + "._C")
    return module
