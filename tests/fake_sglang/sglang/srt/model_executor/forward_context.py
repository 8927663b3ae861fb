"""The forward context the plugin reads (a test stand-in): set ``BACKEND`` / ``POOL``."""

BACKEND = None
POOL = None


def get_attn_backend():
    return BACKEND


def get_token_to_kv_pool():
    return POOL
