"""Parallelism: tensor-parallel target (sharding, fused NVLink collectives, worker protocol).

Data parallelism over independent sessions lives in ``serving.sessions``.
"""
