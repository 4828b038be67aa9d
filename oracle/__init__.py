"""CPU oracle for the Decision Transformer attention path -- TEST INFRASTRUCTURE.

This package is a float32 PyTorch-on-CPU restatement of the reference
algorithm (FujiM3/RL_for_Mario, model/model_decision_transformer.py).  It is
the checker for the CUDA kernels: only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py`` may import it.  The product package
(``rl_for_mario_b200``) never imports or calls it and has no CPU fallback.

Parity pin: the restatement is checked against golden vectors produced by
running the reference module itself (tests/golden/make_golden.py, committed
fixtures tests/golden/*.npz, test tests/test_oracle_golden.py).
"""
from .attention_ref import (  # noqa: F401
    apply_rotary_pos_emb,
    attention_decode_ref,
    attention_module_ref,
    attention_prefill_ref,
    mask_from_pad_len,
    precompute_freqs_cis,
    repeat_kv,
    rmsnorm_ref,
    rotate_half,
)
