"""Stand-in for ``mlx_lm.models.cache``: a plain KV cache type and the
prompt-cache factory the reference's cache factories call."""


class KVCache:
    def __init__(self):
        self.offset = 0


def make_prompt_cache(model, max_kv_size=None):
    n = len(model.layers)
    return [KVCache() for _ in range(n)]
