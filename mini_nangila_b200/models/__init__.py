from .gpt2 import GPT2, GPT2Config
from .llama import Llama, LlamaConfig
from .tinygpt import TinyGPT

__all__ = ["GPT2", "GPT2Config", "Llama", "LlamaConfig", "TinyGPT"]
