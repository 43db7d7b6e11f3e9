"""Plain PyTorch references (fp32/fp64) of every kernel in ``csrc/``.

They are the numerics oracles of the GPU tests and the CPU execution path of
the engine (tests run the whole engine on CPU through them).  Nothing here is
tuned for speed.
"""
