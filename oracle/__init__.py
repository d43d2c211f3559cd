"""CPU oracle for the cirrus-s-1a decode path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithm that the B200
kernels implement, so that the tests can check the GPU results against it.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline.  The product package
(``cirrus_s_1a_b200``) never imports it and has no CPU fallback.

Modules
-------
``nvfp4``    numpy E2M1 / E4M3 codecs, block quantiser, standard packing and
             dequantisation (the format of ``cirrus/perf/bench_kernels.cu:141-145``
             and the dequant of ``scripts/bench_spark.py:290-296, 400-404``).
``indexer``  numpy lightning-indexer scores in a fixed float32 operation order
             and the stable top-k rule of ``cirrus/model/layers.py:282-309``.
``model``    torch-CPU restatement of ``CirrusModel.forward``
             (``cirrus/model/model.py:99-176``) and its layers
             (``cirrus/model/layers.py:33-339``), with optional storage casts
             (bf16 K/V, fp8 E4M3 indexer keys) that the B200 cache uses.

Pinning: ``tests/golden/make_golden.py`` runs the reference model itself (in a
container that has it) and stores its outputs as fixtures; ``tests/test_oracle.py``
checks this oracle against those fixtures.
"""
