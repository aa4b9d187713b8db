"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the W4A16 GEMV path (numpy and C
restatements of the reference's algorithm).  Imported by tests/, the smoke check and
bench.py's CPU-baseline leg; never by the library."""
