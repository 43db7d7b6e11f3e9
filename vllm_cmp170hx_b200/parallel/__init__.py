"""Process groups and collectives (NCCL over NVLink for data, gloo for control)."""
