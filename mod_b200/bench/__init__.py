"""Benchmark harness modules (kernel microbenchmarks, roofline helpers)."""
