"""CPU oracle for the decision-model forward hot path.  TEST INFRASTRUCTURE ONLY.

This package is a plain-PyTorch (CPU, float32/float64) restatement of the arithmetic that the
reference's forward pass runs.  The reference (FastDecisions, ``src/decider``) keeps no model math
of its own: ``decider.engine.Engine._fwd_eager`` (engine.py:115-117) calls the third-party
``transformers`` Qwen3.5 text model.  The pinned third-party version in this image is
transformers 5.5.0, module ``transformers/models/qwen3_5/modeling_qwen3_5.py``; every function
below cites the line of that module (written ``[tf]:line``) or of the reference file it restates.

Pinning: ``tests/golden/make_golden.py`` runs the real transformers 5.5.0 modules (and the
reference's own formulas where they exist) on seeded inputs and stores inputs and outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks every oracle function against those
fixtures.  The oracle is therefore pinned to transformers 5.5.0.  The reference itself pins
transformers 5.17.0 (benchmarks/benchmark.py:548); parity against that version is unpinned.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this package.  The product (``fastdecisions_b200``) never calls it: it has no CPU fallback.
"""

from .ops import (  # noqa: F401
    l2norm,
    residual_rmsnorm,
    rmsnorm_offset,
    packed_conv_silu,
    gdn_gates,
    gated_rmsnorm,
    chunk_gated_delta_rule,
    recurrent_gated_delta_rule,
    rope_cos_sin,
    apply_partial_rope,
    gqa_attention_varlen,
    swiglu,
    slot_readout,
)
