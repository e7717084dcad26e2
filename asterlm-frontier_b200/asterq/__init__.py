"""asterq: B200 (sm_100a) kernels for AsterLM's Hadamard-INT4 latent-cache decode.

Modules (each mirrors one piece of the reference's Python API):
  kv          quantize_tensor / dequantize_tensor / normalized_fwht (quantization/kv.py)
  cache       LatentLayerCache / AsterCache on paged pools (cache.py)
  attention   absorbed decode / causal q_len>1 attention (layers/latent_attention.py)
  decode      batched split-KV decode over paged pools (the C ABI's asterq_latent_decode)
  plan        ragged-batch schedule (tiles, work items, combine jobs)
  sharding    sequence sharding across GPUs
  context_parallel  one long sequence split by chunk across GPUs, partials gathered over NCCL
  synth       seeded synthetic workloads with the benchmark configs' shapes
"""

__version__ = "0.1.0"
