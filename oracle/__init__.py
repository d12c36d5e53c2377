"""CPU oracle for bml's attention / KV-cache path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this package; the CUDA library never calls it.
"""
from .oracle import *  # noqa: F401,F403
