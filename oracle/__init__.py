"""Oracle (test infrastructure only): CPU/FP32 restatements of the reference's
attention formula.  Importable only from tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg; never from the fa_b200 product package."""
