"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the tiered Mamba2 decode state op.

This package is a CPU (torch eager) restatement of nested_ssm's tiered
"dense-but-stale" decode state update. It exists to check the CUDA path and to
serve as the timed CPU baseline. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) may import
it, and only as the checker or the baseline -- never as the thing measured or
shipped. The product package ``nested_ssm_b200`` never imports it.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own code
(``scale/v4_native_decode.py`` through a tiny NemotronH model, and
``scale/vllm_v4_patch.py`` through a stub mixer) and commits its inputs and
outputs as fixtures; ``tests/test_oracle_golden.py`` checks this oracle
against them.
"""
from .tiered import *  # noqa: F401,F403
from .scan import *  # noqa: F401,F403
