"""CPU oracle for the FlashMap drafter hot path (test infrastructure only).

This package restates, on the CPU, the algorithm of the reference FlashMap
drafter (al-jshen/flashmap v0.2.1, ``flashmap/modeling_flashmap.py``): the
one- and multi-jump draft, ``extend_context``, draft sampling and the
acceptance step of ``spec_generate``.  It exists to check the CUDA path; it
is never the thing measured or shipped.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.

Parity pin: the restatement is checked bit-for-bit against golden vectors
that ``tests/golden/make_golden.py`` produced by running the reference code
itself on the CPU (``tests/test_oracle_golden.py``).
"""
