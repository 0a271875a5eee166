"""CPU oracle for the fused single-query decode-attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
/ ``--impl reference`` legs of ``bench.py`` may use it, and there only as the
checker or as the timed CPU baseline, never as the thing measured on the GPU.

Contents
--------
``oracle.quant``      numpy restatement of the reference's per-token symmetric
                      int8 / int4 quantizers and the int4 nibble packer and
                      dequantizer (bit-exact fp16 semantics).
``oracle.attention``  float64 restatement of single-query attention, its GQA
                      head mapping, the split-K partial / log-sum-exp combine
                      algebra, and the reference's torch CPU SDPA path used as
                      the timed CPU baseline.

Parity pin: the restatements are checked against golden vectors produced by
running the reference's own Python functions (``tests/golden/make_golden.py``)
in ``tests/test_oracle_golden.py``.
"""
