"""CPU oracle for the AudioVAE2 decoder hot path: TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this package. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` use it,
and only as the checker (or the timed CPU baseline), never as a code path of
the CUDA decoder.

* ``oracle.decoder``: fp32 restatement of the reference's explicit decoder
  (``src/fast_audiovae/mps_decoder.py``), batch and stateful streaming.
* ``oracle.int8_recipe``: restatement of the reference's W8A8 matrix recipe
  (``experiments/intel-precision/native/precision.cpp``) and the decoder with
  that recipe applied to the "int8_large" matrices.
* ``oracle.reference``: loaders for the real reference code (its Python decoder
  and its compiled C sources under ``oracle/_ref``) used to pin the
  restatements; available only where the reference sources are present.

Parity is pinned: ``tests/golden`` holds vectors produced by the reference's
own decoder and its compiled int8 core (see ``tests/golden/make_golden.py``).
"""
