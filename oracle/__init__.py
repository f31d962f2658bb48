"""CPU oracle: a numpy restatement of the reference's torch f32 decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference leg may import this package, and only
as the checker or the timed CPU baseline -- never as part of the product path
(the B200 backend raises when its CUDA library is missing; it never falls
back here).

Every function cites the reference file:line it restates (paths inside the
breezetoken project).  The oracle is pinned by ``tests/test_oracle.py``
against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``): bit-exact dequantisation vectors, per-op
outputs, and greedy token ids plus logits of full decode runs.
"""
