"""Diagnostics and runtime helpers: device-timed light timing, execution traces and serial trace
export, kernel-call capture, memory attribution and KV plan logging, host-side state index checks."""
