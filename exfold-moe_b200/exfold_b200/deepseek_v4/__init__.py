"""DeepSeek-V4 ExFold ops (drop-in for exfold.deepseek_v4.cuda_ops)."""
