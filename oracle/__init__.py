"""CPU oracle for the polar_pack quad/dual decode path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``polar_pack_b200`` imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
reference legs of ``bench.py`` use it, and there only as the checker or as the
timed CPU baseline -- never as the thing measured or shipped.

Every function restates one piece of the reference's algorithm in numpy and
cites the reference file:line it follows.  Parity of this oracle is pinned by
``tests/test_oracle_golden.py`` against fixtures that
``tests/golden/make_golden.py`` produced by running the reference itself
(its packers, its numpy unpackers, and its Triton kernels under the Triton CPU
interpreter) on seeded inputs.
"""
