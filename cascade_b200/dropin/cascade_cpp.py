"""Import shim: put this directory on PYTHONPATH and ``import cascade_cpp``
(as the reference's ``cascade`` package and adapters do) resolves to
cascade_b200.cascade_cpp."""
import os
import sys

_root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _root not in sys.path:
    sys.path.insert(0, _root)

from cascade_b200.cascade_cpp import *  # noqa: E402,F401,F403
from cascade_b200.cascade_cpp import __all__  # noqa: E402,F401
