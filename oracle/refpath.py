"""Location of the reference source tree — TEST INFRASTRUCTURE.

Used only to build the checker (oracle/Makefile) and the drop-in shim, and by the CPU tests that
compile against the reference's headers.  The tree is the environment variable WUBU_REFERENCE if
set, else the default recorded in oracle/Makefile; None when neither holds a ``src/`` directory
(as on a machine that only runs the prebuilt files).
"""
from __future__ import annotations

import os
import re
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_root() -> Optional[str]:
    path = os.environ.get("WUBU_REFERENCE")
    if not path:
        with open(os.path.join(HERE, "Makefile")) as f:
            for line in f:
                m = re.search(r",([^,()]+)\)\s*$", line)
                if line.startswith("REF ?=") and m:
                    path = m.group(1).strip()
                    break
    return path if path and os.path.isdir(os.path.join(path, "src")) else None
