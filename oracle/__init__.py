"""CPU oracle for the LTHC interface (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and its ``--impl reference`` arm) may import this package.
The product path in ``flowmatching_lthc_b200`` never does.
"""
