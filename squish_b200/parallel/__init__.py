"""Multi-GPU execution: tensor-parallel sharding, NVLink peer-memory collectives, launch helpers."""
