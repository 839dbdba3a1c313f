"""CPU oracle for the Lumina decode path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's CPU algorithm for the decode
hot path (Lumina packed-weight dequant GEMV, KV append/gather, single-query
attention, the dense decode layer and its greedy drivers). Every function cites
the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import it, and only as the checker or the timed CPU
baseline. The product path (``lumina_b200`` + ``liblumina_cuda.so``) never
imports, calls or falls back to anything in here.

Parity pin: the restatement is checked against golden vectors produced by the
reference's own code (``tests/golden/make_golden.py`` imports the reference's
``ptq_ladder``, ``lumina_convert``, ``adapters.lumina``, ``chat``, ``eagle``,
``spec`` and ``tops`` modules and stores their outputs as fixtures).
"""
