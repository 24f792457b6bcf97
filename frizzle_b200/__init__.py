"""frizzle_b200: Frizzle's Gemma 3 1B Q4_0 forward pass and neuron-steering hook as
sm_100a CUDA kernels behind a C ABI (include/frizzle_b200.h).

Submodules: ``engine`` (Device/Model/Batch/generate over the C ABI),
``edits`` (the steering edit table), ``gguf`` and ``synth`` (GGUF files and
seeded synthetic models), ``build`` (nvcc build of the library).
"""

__all__ = ["engine", "edits", "gguf", "synth", "build"]
