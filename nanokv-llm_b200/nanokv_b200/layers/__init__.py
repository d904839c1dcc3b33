"""Drop-in attention modules (reference: nanokvllm/layers, KvChat/layers)."""
