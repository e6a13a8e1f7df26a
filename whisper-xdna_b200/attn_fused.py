"""Drop-in for the reference's src/attn_fused.py entry point attn_head (see
wxb200.attn)."""
from wxb200.attn import attn_head, attn_heads  # noqa: F401
