"""Utilities: kernel microbenchmarks (kernel_bench), device status helpers."""
