"""B200-native LLM serving framework: paged NVFP4/FP8 KV pools, continuous batching with decode burst, speculative
decoding, DSA sparse MLA + MoE and dense GQA model families, hand-written sm_100a kernels, and peer-memory collectives
over NVLink 5.  Import `inference_optimizations_b200.engine` for the serving API."""

__version__ = "0.1.0"
