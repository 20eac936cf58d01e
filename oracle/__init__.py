"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the quantized matvec path (see oracle.py and
qmv_oracle.c).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import it."""
