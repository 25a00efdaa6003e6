from .gpt import GPT, Block, Embedding, GPTConfig, LMHead, build_pipeline_layers

__all__ = ["GPT", "Block", "Embedding", "LMHead", "GPTConfig", "build_pipeline_layers"]
