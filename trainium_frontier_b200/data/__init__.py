"""Synthetic corpus, packing loaders and the byte-length table."""
from .synthetic import BOS_ID, SyntheticTokenizer, get_token_bytes  # noqa: F401
from .loader import PackedRowLoader, make_dataloader, make_eval_dataloader  # noqa: F401
