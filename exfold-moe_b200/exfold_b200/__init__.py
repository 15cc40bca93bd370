"""ExFold routing transform for NVIDIA B200 (sm_100a).

Drop-in modules mirroring the reference's Python API:
  exfold_b200.qwen3.kernels        project_prefill_topk, reroute_decode_subset,
                                   remap_decode_static, select_and_reroute_decode
  exfold_b200.deepseek_v4.cuda_ops torch.ops.dsv4_exfold.{prefill,decode}, fold_prefill,
                                   fold_decode
  exfold_b200.qwen3.router         make_router: the Qwen3 vLLM routing function
  exfold_b200.deepseek_v4.router   make_router: the DeepSeek-V4 vLLM routing function
B200-native entry points: exfold_b200.ops (router, fused router+fold, decode, moe_align, the
grouped SwiGLU expert layer), exfold_b200.parallel (sharded decode over a process group),
exfold_b200.calibration (calibration tables and PairwiseScalarStats).
"""

__version__ = "0.1.0"
