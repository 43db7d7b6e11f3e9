"""Storage-backed tables (rows read from a file per step: Engram-style hash embeddings, per-layer
embedding tables)."""
