"""CPU oracle for the tree-training hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` use it, and only as the checker / the timed CPU baseline.

Every function here restates an algorithm of the reference repository
(Jinghui-Wang/tree-training) in numpy and cites the reference file:line it
follows.  The restatement is pinned against golden vectors produced by running
the reference itself (``tests/golden/make_golden.py``).
"""
