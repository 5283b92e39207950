"""CPU oracle for the LazyRecall KV-management hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (code_for_iclr27_b200) may
import, call or link anything under oracle/.  Only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline / reference legs use it, and
only as the checker or the timed CPU baseline, never as the thing measured.

Pinning: oracle/lrk_oracle.py restates the reference's algorithms in numpy.
It is checked against golden fixtures in tests/golden/, produced by running
the reference itself: its Python CPU path (imported from the reference
source tree) and its own CUDA operators built from its sources by
oracle/build_ref.py into oracle/_ref/.  tests/golden/make_golden.py writes
both kinds of fixture.
"""
