"""CPU oracle (test infrastructure): numpy restatement of the reference's
quantized-GEMM arithmetic. Imported only by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg."""
