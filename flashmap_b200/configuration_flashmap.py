"""Configuration of a FlashMap drafter, served by the B200 CUDA path.

The field names, defaults and validation errors are the reference's
(``flashmap/configuration_flashmap.py:33-138``) so that a release folder's
``config.json`` loads unchanged; the class is written anew here.
"""

from transformers import PretrainedConfig

# "decoding_error" jump grids at the Qwen3 vocabulary size: for ``n`` steps a
# draft jumps grid[i] -> grid[i + 1], i < n.  Values as in the reference
# (configuration_flashmap.py:11-16); they are data, not code.
DEFAULT_JUMP_GRIDS = {
    "1": [0.0, 1.0],
    "2": [0.0, 0.8172569274902344, 1.0],
    "3": [0.0, 0.8010796308517456, 0.8310279846191406, 1.0],
    "4": [0.0, 0.7906050682067871, 0.8172569274902344, 0.8379518389701843, 1.0],
}
MLP_TYPES = ("gelu", "swiglu")
# settings a converted release may name; only these values are served
# (configuration_flashmap.py:19)
FIXED_SETTINGS = {"sampler": "flow_map", "state_featurization": "posterior_noise"}


def jump_times(grid) -> list:
    """``(s, t, next)`` for every jump over ``grid`` (configuration_flashmap.py:22-30).

    A jump evaluates the map from ``s`` to ``t`` and the state then moves to
    ``next``; each jump lands where the next one starts, so ``t == next``.
    """
    points = [float(g) for g in grid]
    return [(a, b, b) for a, b in zip(points[:-1], points[1:])]


class FlashMapConfig(PretrainedConfig):
    """A FlashMap drafter: a DiT flow map that jumps from Gaussian noise over
    the target's vocabulary to a block of ``block_size`` per-slot token
    distributions, conditioned on the target's hidden states.

    Arguments and defaults follow ``FlashMapConfig.__init__``
    (configuration_flashmap.py:82-138): ``target_hidden_size``, ``vocab_size``,
    ``state_vocab_size`` (``None`` = the whole vocabulary, else the size of
    the ``draft_ids`` subset), ``target_layer_ids``, ``block_size``,
    ``hidden_size``, ``num_hidden_layers``, ``num_attention_heads``,
    ``intermediate_size``, ``mlp_type`` ("gelu" or "swiglu"), ``cond_dim``,
    ``time_embed_dim``, ``time_scale``, ``rope_theta``, ``rms_norm_eps``,
    ``qk_norm_eps``, ``layer_norm_eps``, ``noise_gate`` ("jump" or
    "constant"), ``time_schedule``, ``num_steps`` and ``jump_grids``.
    """

    model_type = "flashmap"

    def __init__(
        self,
        target_model: str = "Qwen/Qwen3-8B",
        target_hidden_size: int = 4096,
        vocab_size: int = 151936,
        state_vocab_size=None,
        target_layer_ids=(1, 9, 17, 25, 33),
        block_size: int = 16,
        hidden_size: int = 2048,
        num_hidden_layers: int = 6,
        num_attention_heads: int = 16,
        intermediate_size: int = 8192,
        mlp_type: str = "gelu",
        cond_dim: int = 256,
        time_embed_dim: int = 256,
        time_scale: float = 1000.0,
        rope_theta: float = 10000.0,
        rms_norm_eps: float = 1e-6,
        qk_norm_eps: float = 1e-5,
        layer_norm_eps: float = 1e-6,
        noise_gate: str = "jump",
        time_schedule: str = "decoding_error",
        num_steps: int = 1,
        jump_grids=None,
        **kwargs,
    ):
        if state_vocab_size is not None and not 0 < int(state_vocab_size) <= vocab_size:
            raise ValueError(f"state_vocab_size must be in (0, {vocab_size}], got {state_vocab_size}")
        if mlp_type not in MLP_TYPES:
            raise ValueError(f"mlp_type must be one of {MLP_TYPES}, got {mlp_type!r}")
        for name, allowed in FIXED_SETTINGS.items():
            if kwargs.pop(name, allowed) != allowed:
                raise ValueError(f"this version of flashmap serves only {name}={allowed!r}")
        self.target_model = target_model
        self.target_hidden_size = target_hidden_size
        self.vocab_size = vocab_size
        self.state_vocab_size = None if state_vocab_size is None else int(state_vocab_size)
        self.target_layer_ids = list(target_layer_ids)
        self.block_size = block_size
        self.hidden_size = hidden_size
        self.num_hidden_layers = num_hidden_layers
        self.num_attention_heads = num_attention_heads
        self.intermediate_size = intermediate_size
        self.mlp_type = mlp_type
        self.cond_dim = cond_dim
        self.time_embed_dim = time_embed_dim
        self.time_scale = time_scale
        self.rope_theta = rope_theta
        self.rms_norm_eps = rms_norm_eps
        self.qk_norm_eps = qk_norm_eps
        self.layer_norm_eps = layer_norm_eps
        self.noise_gate = noise_gate
        self.time_schedule = time_schedule
        self.num_steps = num_steps
        self.jump_grids = dict(DEFAULT_JUMP_GRIDS if jump_grids is None else jump_grids)
        kwargs.setdefault("tie_word_embeddings", False)
        super().__init__(**kwargs)


__all__ = ["DEFAULT_JUMP_GRIDS", "FlashMapConfig", "jump_times"]
