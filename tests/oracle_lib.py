"""Test-side access to the CPU oracle (oracle/oracle_ctypes.py)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
from oracle_ctypes import *  # noqa: F401,F403,E402
from oracle_ctypes import load_oracle, ptr, f32, rel_l2  # noqa: F401,E402
