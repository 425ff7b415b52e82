"""B200-native attention path for the alpaccaroo inference engine.

Layers:
  include/b2attn.h, csrc/     C ABI + sm_100a CUDA kernels (libb2attn.so)
  _lib                        ctypes binding, status -> exception mapping
  device                      device-tensor API (torch tensors as carriers)
  kernels, cuda, qwen35_kernels
                              drop-ins with the reference's Python signatures
                              (alpaccaroo/kernels.py, cuda.py, qwen35_kernels.py)
  model_hooks                 installs the drop-ins on an alpaccaroo Model
  kvstate                     device-authoritative attention state with the
                              reference's snapshot records; host-mirror semantics
  decode_step                 one batched decode step (RoPE + append + decode)
                              replayed as a CUDA graph
  longctx                     long-context decode split across GPUs
  qwen35_layer                Qwen35 full-attention layer step on the device
  decode_chain, prefill_chain whole decode token / prefill chunk of a Q8_0 llama
                              model on the device
"""
from . import _lib  # noqa: F401
from ._lib import B2AError, B2AShapeError, B2ADeviceError  # noqa: F401

__all__ = ["B2AError", "B2AShapeError", "B2ADeviceError"]
