"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the ring-attention hot path.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg (and its
``--impl reference`` arm) may import it.  The product package (``fa4_ring``
under ``fa4-cp_b200/``) never imports anything from here and has no CPU
fallback.

``ring_oracle`` restates, in numpy, the reference's CPU algorithm for the path
(hxy0118/fa4-cp): the zig-zag index math of ``fa4_ring/zigzag.py`` and the
per-chunk attention / online-softmax merge / ring simulation of
``tests/test_algorithm_cpu.py``.  It is pinned against golden vectors produced
by importing the reference itself (``tests/golden/make_golden.py``).

``bwd_oracle`` is the gradient of that forward (the reference itself is forward-only),
pinned against torch autograd through the reference's dense forward.
"""
