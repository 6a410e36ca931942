"""kdev problem reference for the fused MoE layer, moe_prefill configuration.  TEST INFRASTRUCTURE:
the reference module kdev imports; body in oracle/problems/moe_problem.py."""
import sys
from pathlib import Path

_HERE = Path(__file__).resolve().parent.parent
if str(_HERE) not in sys.path:
    sys.path.insert(0, str(_HERE))

from moe_problem import make  # noqa: E402

globals().update(make("moe_prefill"))
