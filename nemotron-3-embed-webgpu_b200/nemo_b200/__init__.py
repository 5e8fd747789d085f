"""B200-native Nemotron-3-Embed-1B encoder: Python host side.

``runtime`` binds the CUDA library (libnemo_b200.so) through its C ABI,
``engine`` restates the reference's micro-batching embedding engine, ``synth``
makes seeded synthetic ``.wgpack`` models and inputs, ``wgpack`` writes the
container format.
"""
from .engine import NemotronEmbeddingEngine  # noqa: F401

__all__ = ["NemotronEmbeddingEngine"]
