"""models package."""
from .gpt import GPT, Block, CausalSelfAttention, MLP  # noqa: F401
