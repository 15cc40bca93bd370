"""Qwen3 ExFold routing functions (drop-in for exfold.qwen3.kernels)."""
