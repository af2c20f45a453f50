"""CPU oracle package (test infrastructure only: tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs use it as the checker; the product never imports it)."""
