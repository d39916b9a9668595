"""CPU oracle of the FPN neck -- test infrastructure only (see fpn_oracle.py).

Importable by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference arms; never by the library."""
