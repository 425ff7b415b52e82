"""CPU oracle for the B200 attention path - TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy and plain Python, the reference's CPU
algorithms for the three hot-path ops (decode attention, causal prefill
attention, RoPE + KV append) plus the split-KV combine.  Each function cites
the reference file:line it follows (paths inside the alpaccaroo project).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import it, and only as the checker or the timed CPU baseline.  The product
path (alpacca_open_sourced_by_jt_b200) never imports it and has no CPU
fallback.

Parity pinning: tests/golden/*.npz hold outputs of the reference itself
(alpaccaroo, run in the build container by tests/golden/make_golden.py on
seeded inputs); tests/test_oracle.py checks this oracle against them.
"""
from .attention import (  # noqa: F401
    attention_decode,
    attention_batch,
    attention_decode_varlen,
    split_decode_partials,
    split_combine,
    lse_combine,
    qwen35_full_attention_decode,
    qwen35_full_attention_prefill,
    causal_gqa_step,
)
from .rope import (  # noqa: F401
    rope_inv_freq,
    rope_tables,
    rope_vec,
    rope_batch,
    rope_append,
    imrope_lane_for_pair,
    imrope_rotate,
    imrope_append,
)
from .qwen35_layer import (  # noqa: F401
    qwen35_rms_norm,
    qwen35_attention_layer,
)
from . import llama_q8  # noqa: F401
