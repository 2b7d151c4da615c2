"""CPU oracle for the continuous-batching decode path — TEST INFRASTRUCTURE ONLY.

This package restates the reference's algorithm (qweninfer, Python/PyTorch) in plain
numpy float32 so that the CUDA path can be checked against it on machines where the
reference itself is not installed. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it, and only as the
checker or the timed CPU baseline. The product package `qweninfer_b200` never imports
it and has no CPU fallback.

Pinning: `tests/test_oracle_golden.py` checks this oracle against golden vectors that
`tests/golden/make_golden.py` produced by running the reference package itself on the
same seeded weights and inputs.
"""

from oracle.qwen2_ref import (  # noqa: F401
    OracleCache,
    OracleModel,
    bf16_round,
    build_rope_cache,
    load_safetensors_fp32,
    oracle_generate,
    rmsnorm,
)
from oracle.engine_ref import OracleEngine, OracleRequest  # noqa: F401
