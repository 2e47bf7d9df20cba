"""CPU oracle for the drafter training step -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the reference's drafter
training step (``pe.partition.mtp_backward`` and everything it calls) and its
draft-time path (``draft_logits`` and the tree / chain proposals).  It is the
checker that the CUDA path is compared against, and the "port" timed as the CPU
baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it; the product package never does, and has no CPU
fallback.

Parity pin: the restatement is checked against golden vectors produced by running
the reference itself (``tests/golden/make_golden.py``), see
``tests/test_oracle_golden.py``.
"""

from .drafter_step import (  # noqa: F401
    OracleDims,
    attention,
    attention_flops,
    count_loss_slots,
    drafter_forward,
    init_params,
    mask_input,
    mtp_eval_loss,
    mtp_step,
    param_names,
    real_input,
    rms_norm,
    rope_tables,
    segment_edges,
    segment_slots,
    slot_allow,
)
from .draft import (  # noqa: F401
    draft_logits,
    draft_logits_sequential,
    propose_chain_from_logits,
    propose_tree_from_logits,
    token_shared_input,
    tree_allow,
    tree_positions,
)
