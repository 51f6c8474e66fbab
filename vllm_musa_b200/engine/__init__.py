"""Serving engine: LLMEngine, model runner (CUDA graphs), step buffers."""
