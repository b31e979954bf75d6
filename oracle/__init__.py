"""CPU oracle for the Mamba-3 trapezoidal selective scan and its O(1) step.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped product path imports this
package: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg (``cpu_baseline`` / ``--impl reference``) use it, and only as the
checker or as the timed CPU baseline, never as the thing measured on the GPU.

The oracle restates, in plain PyTorch on the CPU, the reference algorithm of
PranavPrasannaV/RedPanda ``redpanda/engine/mamba.py`` (the chunked
Hillis-Steele trapezoidal scan and ``Mamba3Block.step``).  Every function cites
the reference lines it follows.  It is pinned against golden vectors that were
produced by running the reference module itself (``tests/golden/make_golden.py``
imports the read-only reference and writes ``tests/golden/*.pt``); the CPU test
``tests/test_oracle_golden.py`` checks the restatement against them.
"""

from .scan_oracle import (  # noqa: F401
    SCAN_CHUNK,
    compute_A,
    track_gate,
    pad_params,
    parallel_scan,
    scan_chunked,
    scan_sequential,
    scan_bidir,
    scan_with_grads,
    step_cells,
)
from .model_oracle import (  # noqa: F401
    OracleConfig,
    block_forward,
    block_step,
    model_forward,
    model_step,
    model_prime_cache,
)
