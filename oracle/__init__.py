"""Test infrastructure: the CPU FP32 oracle the CUDA path is checked against.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package.  The product (``tiktoktechjam2026_b200``)
never does.  See ``oracle/reference_fp32.py`` for what it restates and where
each function comes from in the reference.
"""

from .reference_fp32 import (  # noqa: F401
    ATOL,
    CONFIGS,
    DEFAULT_SEED,
    RTOL,
    SUITE_CONFIGS,
    TIMING_SEED_OFFSET,
    Comparison,
    Config,
    compare,
    forward,
    forward_flops_bytes,
    generate_case,
    pack_qkv_state_dict,
    seeded_state_dict,
)
