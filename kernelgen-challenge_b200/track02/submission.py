"""Drop-in ``submission.py`` for the reference's track-02 harness.

The harness (track-02/test_correctness.py:12-13, bench.py:14) does
``from submission import hc_split_sinkhorn``; put this directory first on
``sys.path`` (its parent holds the ``sparse_attn`` package).
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from sparse_attn.mhc import hc_split_sinkhorn  # noqa: E402,F401

__all__ = ["hc_split_sinkhorn"]
