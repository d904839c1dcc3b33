"""nanokv_b200: B200 (sm_100a) kernels for nano-kvllm's attention hot path.

The CUDA code lives in libnkv.so (C ABI, include/nkv.h); `ops` wraps it for
torch tensors, `layers` mirrors the reference's Attention modules, `utils`
its Context contract and `engine` the host-side compression metadata
(selection, events, block truncation). Build the library with
`python -m nanokv_b200.build`.
"""

__all__ = ["ops", "build"]
