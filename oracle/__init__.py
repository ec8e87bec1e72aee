"""CPU oracle for the GGUF quantized-matmul path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this package, and only as the checker / the timed reference CPU path.  The
product (``rce_b200``) never imports it.
"""
from .oracle import *  # noqa: F401,F403
