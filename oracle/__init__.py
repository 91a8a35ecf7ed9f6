"""CPU oracle for the Qwen3.6-35B-A3B MoE block hot path -- TEST INFRASTRUCTURE ONLY.

Nothing under this directory is part of the product. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import, link or run it, and only as the checker (or as the timed CPU
restatement of the reference's own CPU path). The CUDA path never calls into it and
fails loudly when its extension is missing.

Contents, each function citing the reference file:line it restates:

* ``q4k``     -- GGUF Q4_K super-block layout, ``get_scale_min_k4`` and its inverse, the
                 f64-exact dequant (``tools/gguf_reader.py:165-176, 248-267``), and a numpy
                 mirror of the seeded synthetic block generator the device uses.
* ``bf16``    -- bf16/f16 bit helpers (round-to-nearest-even, as torch ``.to(bfloat16)``).
* ``moe``     -- the MoE block: router R1-R5 under the declared deterministic order
                 (through the C restatement in ``c/oracle.c``), an f64 block restatement of
                 ``engine/m3_forward.py:430-476``, and a torch-f32 port of the same function
                 used as the timed CPU baseline.
* ``c/``      -- plain-C restatement of the bit-exact parts (dequant, router, RMSNorm)
                 compiled by ``build.py`` with gcc into ``oracle/_build/liboracle.so``.

Parity pins: ``tests/golden/make_golden.py`` imports the reference's own Python
(``tools/gguf_reader.py``, ``tools/gguf_fast_dequant.py``, ``engine/m3_forward.py``)
in the build container and writes the fixtures under ``tests/golden/`` that
``tests/test_oracle_golden.py`` checks this oracle against.
"""
