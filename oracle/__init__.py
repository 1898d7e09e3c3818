"""CPU oracle for the GGUF weight-preparation path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline / reference arm of ``bench.py`` may import this package, and only as the
checker or as the timed CPU baseline.  The product path (``llima_b200``) never
imports it and has no CPU fallback.
"""
