"""CPU oracle for the fused RMSNorm + RoPE path (test infrastructure only).

This package restates, in plain PyTorch on the CPU, what the reference
(shell-bay/bloth) computes on this path. It is the checker that the CUDA
kernels are compared against, and the timed CPU baseline of ``bench.py``.
Nothing in the product (``bloth_b200``) imports it.

Pinned against golden vectors produced by running the reference's own Triton
kernels under the Triton CPU interpreter (``tests/golden/make_golden.py``);
``tests/test_oracle.py`` checks the restatement against them.
"""
from .reference_path import (  # noqa: F401
    inv_freq,
    rope_cos_sin,
    rms_norm,
    rms_norm_fwd_bwd,
    add_rms_norm_fwd_bwd,
    norm_rope_table,
    norm_rope_table_fwd_bwd,
    norm_rope_table_reference_bwd,
    qk_norm_rope,
    qk_norm_rope_fwd_bwd,
    rope,
    rope_fwd_bwd,
    packed_position_ids,
    rms_norm_dw_scale,
    rms_norm_dx_scale,
    qk_dw_scale,
    norm_rope_table_dw_scale,
    qk_dx_scale,
    tolerance_ok,
)
