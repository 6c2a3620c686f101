"""Command-line tools kept flag-compatible with the reference's llk-compile,
llk-bench and llk-tune, plus micro-perf (``python -m dslcompiler_b200.cli.<tool>``)."""
