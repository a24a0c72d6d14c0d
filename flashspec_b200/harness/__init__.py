"""Measurement harness: microbench (single point), profile_matrix (sweeps) and ncu_parse."""
