"""CPU oracle for scree's varlen hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithms (jvoltci/scree,
src/scree/_core.py and src/scree/kernels/reference/*.py), used as the checker
for the CUDA kernels of scree_b200.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm may import it; the product path
(scree_b200) never does.

Pinning: every function here is checked against golden vectors produced by
running the real reference (tests/golden/make_golden.py imports it from a
local checkout and stores inputs + outputs as fixtures), see
tests/test_oracle_golden.py.
"""

from .varlen import (  # noqa: F401
    attention_bwd,
    attention_fwd,
    from_padded,
    layernorm_bwd,
    layernorm_fwd,
    pack,
    rmsnorm_bwd,
    rmsnorm_fwd,
    softmax_bwd,
    softmax_fwd,
    to_padded,
    unpack,
)
