"""Reported baselines that are not part of the library: the reference's GPU
kernels restated in CUDA C (refkernels.cu, loaded by refkernels.py)."""
