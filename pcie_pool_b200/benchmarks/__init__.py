"""Benchmarks: kernel-level (``land_kernel``) and workload-level runs."""
