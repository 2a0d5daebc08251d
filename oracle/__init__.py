"""CPU oracle for the KV-cache erasure-coding path — TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this package.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs use
it, and only as the checker (or the timed CPU baseline), never as a fallback.

Modules
-------
``reference``  numpy restatement of the reference's own codecs, function by
               function, each citing the file:line it follows:
               XOR (benchmark/xor), mod-S "RDP" (benchmark/rdp and the hook
               extension in bench_ghostserve_rdp.py), Reed-Solomon over GF(2^16)
               (benchmark/rs).
               Pinned against the reference itself: tests/golden holds outputs of
               the reference CUDA extensions (built from the reference sources by
               ``oracle/build_ref.py`` into ``oracle/_ref``) run on a B200 on the
               same host-generated inputs; ``tests/test_golden.py`` checks this
               module against them.
``codes``      numpy implementation of the codes the reference does not have:
               textbook Row-Diagonal Parity (Corbett et al., FAST 2004) with p
               prime and stripe units, and Reed-Solomon over GF(2^8)/0x11d with a
               Cauchy generator.  There is no reference implementation to run, so
               these are pinned by hand-checkable known-answer vectors, algebraic
               properties (MDS: every <= m erasure pattern decodes), a decoder
               written independently of the CUDA decoder (peeling over
               row/diagonal equations, versus precomputed syndrome masks), and
               the SHA-256 digests of a second, independent restatement
               (``tests/golden/kat.py``: bitwise field arithmetic, a diagonal walk)
               committed in ``tests/golden/kat_codes.json``.
``cpu``        C/OpenMP restatement used as the timed CPU baseline (built by
               ``oracle/cpu/Makefile`` into ``oracle/cpu/liboracle.so``).
``build_ref``  recipe that compiles the reference's CUDA extensions into
               ``oracle/_ref`` (git-ignored).
"""
