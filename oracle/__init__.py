"""CPU oracle for the int4 MatMulNBits linear path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this directory; only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of ``bench.py``
may use it, and only as the checker or as the timed CPU baseline, never as a GPU fallback.

Parity pin: ``tests/golden/`` holds fixtures produced by executing the reference's own
``quant()`` function (convert/export_engine.py:17-26, extracted from the source file with
``ast`` and run under torch) and the reference's weight generator statements
(convert/make_gemm.py:4-10, convert/make_chain.py:22-29). ``tests/test_oracle.py`` checks this
restatement against those fixtures bit-exactly.
"""
