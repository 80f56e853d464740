"""CPU oracle for the replica hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of p2pLLM's replica path (p2p/wanda.py, p2p/compact.py, p2p/replica.py, p2p/route.py), each
function citing the reference lines it follows. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
(and its `--impl reference` arm) may import it, and only as the checker or as the timed CPU baseline: the product
path (p2pllm_b200) never calls it.

Pinning: tests/golden/make_golden.py runs the reference's own p2p.wanda / p2p.compact on seeded inputs and commits
their outputs as fixtures; tests/test_oracle_golden.py checks this oracle against them and against the reference's
unit-test vectors (tests/test_wanda.py, tests/test_sglang.py). Where the reference leaves tie order unspecified
(torch.topk), the oracle breaks ties by the lower column, and the fixtures count the rows where that matters.
"""
from .wanda_oracle import (bf16_to_f32, f32_to_bf16, k_of, scores, select, sumsq_cols, channel_norms,  # noqa: F401
                           expert_inputs, prune, tie_rows)
from .compact_oracle import pack, unpack, expand_idx, forward, forward_blocks, words_to_idx  # noqa: F401
from .replica_oracle import combine, summed, member_part  # noqa: F401
