"""ORACLE -- test infrastructure only: CPU restatements used as the checker
(tests, ``__graft_entry__.smoke``) and as the timed CPU baseline in
``bench.py``.  Never imported by the ``phew_b200`` package."""
