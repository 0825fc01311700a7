"""Test infrastructure: the reference's own CPU implementation (oracle/_ref, built from the
reference sources by oracle/Makefile), its numpy restatement (port.py) and ctypes access
(ref.py).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.

REFERENCE_ROOT is where the read-only reference checkout is found when it is present (the
build machine); the GPU box has only the prebuilt oracle/_ref files.  Override it with the
DCB_REFERENCE_ROOT environment variable (oracle/Makefile reads the same variable).
"""
import os

REFERENCE_ROOT = os.environ.get("DCB_REFERENCE_ROOT", "/root/reference")
REFERENCE_SRC = os.path.join(REFERENCE_ROOT, "worker-cuda", "src")
