"""CPU oracle for the top-k sparse attention path (test infrastructure only).

Importable by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py``; the product package never imports it.
"""

from .topk_attention import *  # noqa: F401,F403
