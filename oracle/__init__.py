"""CPU oracle for the FlashAttention-forward and matmul hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this package: only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it,
and only as the checker or the timed CPU reference, never as a code path that
produces results for users.

Contents
  fa_oracle.py   numpy restatement of the reference's tiled online-softmax
                 attention forward (flash_atten.py:14-133 and variants) and the
                 reference's own correctness oracle, torch SDPA on fp32 CPU
                 copies (test_flash_atten.py:459-461, 498-499).
  mma_oracle.py  numpy restatement of the reference matmul (mma.py:8-52) and
                 its oracle, torch.matmul on CPU (test_mma.py:296-297).
  rounding.py    round-to-nearest-even casts to bf16 / fp16 in numpy.

Pinning: tests/golden/ holds input/output vectors produced by running the
reference's own Triton kernels in Triton's CPU interpreter
(tests/golden/make_golden.py); tests/test_oracle.py checks this oracle against
every one of them.
"""
