"""CPU oracle (test infrastructure): restated reference algorithms used only as
the checker in tests/, __graft_entry__.smoke() and bench.py's CPU baseline."""
