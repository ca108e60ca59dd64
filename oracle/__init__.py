"""CPU oracle for the NVFP4 quantizer and simulated-FP4 attention.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
CPU legs of bench.py (``cpu_baseline`` and ``--impl reference``) may import
this package, and only as the checker or the timed CPU baseline.  The
product package ``fp4_attn_b200`` never imports it.

* ``oracle.quant``      -- ctypes face of nvfp4_oracle.c (codes/scales, both
                           reference flavours), bit-exact to the reference.
* ``oracle.torch_port`` -- torch CPU restatement of the quantizer and of the
                           simulated-FP4 attention.

Parity pins: tests/golden/* were produced by running the reference itself
(tests/golden/make_golden.py); tests/test_oracle_golden.py checks both
restatements against them.
"""
