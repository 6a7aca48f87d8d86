"""Where the reference project's checkout is, for the CPU tests that import
its Python package (its evaluator, sequential loop, MCTS, autotuner and
config loader driving this package's backend).

``KMCTS_REFERENCE_ROOT`` names the checkout; unset, the build container's
checkout location is tried.  Tests that need it skip when the directory is
absent, as on a GPU box, where the reference tree does not travel.
"""

from __future__ import annotations

import os
from pathlib import Path

REFERENCE_ROOT = Path(os.environ.get("KMCTS_REFERENCE_ROOT", "/root/reference"))
REFERENCE_SRC = REFERENCE_ROOT / "src"
