"""Per-step Context contract (reference: nanokvllm/utils/context.py)."""
