"""CPU oracle for the nano-kvllm attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU and in plain torch/numpy, what the
reference computes on the path that libnkv replaces:

  * store_kvcache slot writes        (nanokvllm/layers/attention.py:10-40)
  * paged decode attention           (flash_attn_with_kvcache semantics at
                                      nanokvllm/layers/attention.py:104-107)
  * prefill / mixed-batch attention  (flash_attn_varlen_func semantics at
                                      nanokvllm/layers/attention.py:96-102)
  * SnapKV scoring + top-k           (nanokvllm/layers/CompressMethod.py:4-58,
                                      KvChat/layers/CompressMethod.py:4-58)
  * periodic window compression      (nanokvllm/layers/compress_utils.py:9-290)
  * KvChat threshold compression     (KvChat/layers/compress_utils.py:10-171,
                                      :218-252) and its query window
                                      (KvChat/engine/query_window_manager.py)
  * unified-step metadata            (nanokvllm/engine/model_runner.py:154-219)
  * request state and block manager  (nanokvllm/engine/sequence.py,
                                      nanokvllm/engine/block_manager.py): the
                                      stand-ins the host tests drive the
                                      product's event appliers with

It is the checker, never the product: only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg import it. The product (nanokv_b200) never
imports it and has no CPU fallback.

Pinning: the compression restatements are checked against golden vectors
produced by running the reference's own functions on the CPU
(tests/golden/make_golden.py). Decode attention's arithmetic lives in the
third-party flash-attn package (unpinned in the reference's pyproject.toml;
2.8.3 in this image); its restatement is pinned by outputs of
flash_attn_with_kvcache itself recorded on a B200 (tests/golden/make_golden_flashattn.py).
"""
