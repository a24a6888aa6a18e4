"""Utilities: per-phase device timers with NVTX ranges (timers), kernel microbenchmarks
(kernel_bench), the engram module benchmark (engram_bench) and the peer-memory all-reduce
benchmark (p2p_bench)."""
