"""Continuous-batching inference engine: requests, scheduler, cache pools, runner."""
