"""CPU oracle for the KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference engine's algorithms for the
path (paged append, paged decode / varlen / mixed attention, E4M3 codec, page
copy).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
(`--impl reference` and the `cpu_baseline` figure) may import it, and only as
the checker or as the timed CPU baseline.  The product path
(slo-aware-llm-serving-engine_b200/) never imports it and has no CPU fallback.

Parity is pinned: tests/golden/make_golden.py runs the reference's own code
(its Triton store kernel under the interpreter, its fp32 attention oracle, its
E4M3 encoder and its page-restore routine) and commits the outputs as fixtures
under tests/golden/; tests/test_oracle_golden.py checks this restatement
against them.
"""
