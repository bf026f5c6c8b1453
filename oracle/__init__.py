"""CPU oracle for the GDNX recurrent-scan hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``gdnx_b200``) imports
this package; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` use it, and only as the checker or as the timed CPU baseline.

The modules restate, in plain PyTorch on the CPU, the reference's own
recurrences (each function cites the reference ``file:line`` it follows):

* ``recurrence.gdn3_kr_scan``   -- frozen GDN3 Kronecker-residual token loop
  (``gdn3/_reference_recurrence.py:33-94``) that also returns the final state.
* ``recurrence.dense_scan``     -- its dense special case (compaction off),
  ``S_t = g S + a (u - g S h) k^T``, ``y = S_t q``.
* ``recurrence.kmd2_scan``      -- KMD-2 frozen loop
  (``research/kernel_ab/ref_scan.py:24-48``) + update-norm scores
  (``research/kmd2_ablation/exact_cache.py:1231-1295``) + final state.
* ``recurrence.compact_call``   -- one rearrangement-SVD compaction
  (``gdn3/gdn3_upgrade.py:650-719``) with the Gaussian sketch supplied.
* ``recurrence.compact_sketch_call`` -- the ``compact_mode`` "sketch" /
  "sketch_noqr" compaction (``gdn3/gdn3_upgrade.py:579-596``).
* ``prologue``                  -- braided decay and lane RoPE
  (``gdn3/gdn3_upgrade.py:342-401, 809-822``).
* ``inputs``                    -- seeded synthetic inputs for the five
  BASELINE configurations.

Parity pin: ``tests/golden/make_golden.py`` imports the reference from its
source tree, runs it on seeded inputs and stores the outputs as fixtures;
``tests/test_oracle_golden.py`` checks these restatements against them
(bit-exact where the op sequence is identical).
"""
