"""CPU oracle for the INT4 decode path (test infrastructure only).

A ctypes binding over ``oracle/glacier_oracle.c``, the C restatement of the
reference's portable FP32-activation path.  Only the tests, the smoke check in
``__graft_entry__`` and the CPU-baseline legs of ``bench.py`` import this
package; the CUDA library never calls it.
"""
from .oracle import *  # noqa: F401,F403
