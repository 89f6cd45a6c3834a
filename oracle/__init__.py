"""CPU oracle for the snapmind KV-cache hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithms (each function cites the
reference file:line it follows).  Only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py`` may import it, and only as the checker
or as the timed CPU baseline; the ``snapmind_b200`` package never does.

The oracle is pinned against golden vectors produced by running the reference
itself (``tests/golden/make_golden.py``); see ``tests/test_oracle_golden.py``.
"""
