"""Per-card tuning tables (TOML data, see vllm_cmp170hx_b200/tuning_table.py)."""
