"""Pallas-Triton names (stand-in; never called)."""


class TritonCompilerParams:
    def __init__(self, *_a, **_k):
        pass


CompilerParams = TritonCompilerParams
