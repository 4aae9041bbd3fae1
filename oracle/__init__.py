"""ORACLE — test infrastructure only.

CPU restatements of the reference's group-rational path used to check the CUDA library:
kat_torch_oracle (the reference's PyTorch op sequence, fp32 or fp64) and c_oracle (a
float64 C restatement with magnitude sums).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import this package; the library never does.
"""
