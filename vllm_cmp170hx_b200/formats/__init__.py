"""Checkpoint formats: EXL3 trellis, Marlin int4 group-128, fp8 block-scaled."""
