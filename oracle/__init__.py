"""CPU oracle for the per-chunk causal self-attention hot path — TEST INFRASTRUCTURE.

A restatement, in numpy / torch-CPU, of the reference's algorithms on this path
(each function cites the reference file:line it follows).  It is the checker
the GPU parity tests compare against and the CPU baseline the benchmark reports
next to the GPU numbers.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import it; the reworld_b200 package never does.

Pinning: tests/golden/make_golden.py runs the reference itself on CPU and
stores its outputs under tests/golden/; tests/test_oracle_golden.py checks this
oracle against those fixtures (attention, RoPE, landmark-bank decisions and
cache bytes, Ulysses all-to-all layouts).
"""
