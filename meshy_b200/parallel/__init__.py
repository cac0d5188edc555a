"""Parallelism: DDP/FSDP/CP/EP/TP plumbing and the fused NVLink collectives."""
