"""CPU oracle of the decode hot path — TEST INFRASTRUCTURE ONLY.

Only the test suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import this package, and only as the checker or as the timed
CPU baseline. The product path (the ``cscr`` op modules) never calls it.
"""
