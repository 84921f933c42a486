"""Kernel microbenchmarks (roofline fractions against measured peaks)."""
