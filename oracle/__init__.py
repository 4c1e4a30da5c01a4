"""CPU oracle for the Kshipra quantized forward path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``kshipra_b200`` imports this package:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may use it, and only as the checker or as the timed CPU
baseline -- never as a product code path.

What it restates (own code, citing the reference file:line it follows):

* ``oracle.quant``     -- numpy restatement of engine/quantization.py
  (INT8 per-channel, INT4 per-group packing and dequantization).  Byte-exact.
* ``oracle.attention`` -- torch-CPU restatement of engine/chunked_prefill.py
  ``chunked_attention`` / ``monolithic_attention``.
* ``oracle.model``     -- torch-CPU restatement of engine/model.py
  ``KshipraModel.forward`` / ``generate`` (including the HF RMSNorm / SwiGLU
  module arithmetic it calls), working on a plain state dict.

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself
(importing its ``engine`` package in the build container) on seeded inputs and
stores the outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks every function here against those fixtures.
"""
