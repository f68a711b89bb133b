"""The NCA cell rule with the reference's module layout, executed by the B200 kernels.

`NCAConfig` carries every field of nca.model.NCAConfig (src/nca/model.py:48-137) so that configs
and state dicts of the reference load unchanged.  `NCA` has the same parameter names
(`perceive.weight`, `update.fc1`, `update.fc2`, `head`, buffer `embed`) so
`NCA.load_state_dict(reference_model.state_dict())` works, and the same methods as the
reference's NCA on the rollout path: `init_state`, `apply_clamp`, `step`, `sample_fire_mask`,
`scores`, `decode`, `confidence`, `board_confidence`.  Their compute runs in libnca_b200 (see
`ncas_b200.engine`); parameters are plain torch tensors used as storage.

The kernels implement the subset of the reference's cell rules used by the benchmark configs:
4-head KernelPerception with zero padding, the ReLU MLP update, no group normalisation, no
step/task embeddings, and an `mlp` readout head.  Anything else raises ValueError, as the
reference's fast engine does for combinations it lacks (src/nca/engine/step.py:93-125).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import numpy as np
import torch
from torch import nn

# Fixed perception heads of the benchmark models: identity, Sobel-x, Sobel-y, Laplacian.
IDENTITY = [[0.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 0.0]]
SOBEL_X = [[-0.125, 0.0, 0.125], [-0.25, 0.0, 0.25], [-0.125, 0.0, 0.125]]
SOBEL_Y = [[-0.125, -0.25, -0.125], [0.0, 0.0, 0.0], [0.125, 0.25, 0.125]]
LAPLACIAN = [[0.0625, 0.125, 0.0625], [0.125, -0.75, 0.125], [0.0625, 0.125, 0.0625]]
FIXED_TAPS = np.array([IDENTITY, SOBEL_X, SOBEL_Y, LAPLACIAN], dtype=np.float32)


@dataclass
class NCAConfig:
    """Architecture hyper-parameters; same fields and defaults as nca.model.NCAConfig."""

    vocab_size: int
    channels: int
    c_in: int
    c_out: int
    output_tokens: tuple[int, ...]
    in_offset: int = 0
    out_offset: int = 0
    c_task: int = 0
    n_tasks: int = 0
    embedding: str = "onehot"
    perception: str = "kernels"
    heads: int = 4
    grid_size: tuple[int, int] | None = None
    padding: str = "wall"
    wall_token: int | None = 2
    update: str = "mlp"
    expansion: int = 2
    hidden_from_perception: bool = False
    norm_groups: int = 0
    norm_fired_only: bool = False
    sigma_init: float = 0.15
    init_uniform: bool = False
    fire_rate: float = 0.8
    head: str = "l2"
    time_steps: int = 0
    zero_init_update: bool = True
    attn_bias: bool = True
    project_update: bool = False
    noise_after_norm: bool = False
    norm_init: bool = False
    norm_style: str = "sqrt_eps"
    init_style: str = "torch"

    def __post_init__(self) -> None:
        self.output_tokens = tuple(int(t) for t in self.output_tokens)
        c = self.channels
        assert self.in_offset + self.c_in <= c, "input slice exceeds the state"
        assert self.out_offset + self.c_out <= c, "output slice exceeds the state"

    @property
    def in_slice(self) -> slice:
        return slice(self.in_offset, self.in_offset + self.c_in)

    @property
    def out_slice(self) -> slice:
        return slice(self.out_offset, self.out_offset + self.c_out)

    @property
    def perception_dim(self) -> int:
        return self.heads * self.channels

    @property
    def hidden(self) -> int:
        return self.expansion * (self.perception_dim if self.hidden_from_perception else self.channels)

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> NCAConfig:
        return cls(**d)


# (channels, hidden) instances of the step kernel: the benchmark models and the reference's
# maze presets (maze_ood 16/128, maze_hard 32/256)
KERNEL_SHAPES = ((32, 128), (64, 256), (16, 128), (32, 256))

# The reference's maze presets (src/nca/model.py:656-700), the ones whose cell rule the kernels
# implement: learned 4-head 3x3 perception, wall padding, MLP update, l2 head.
PRESETS: dict[str, dict] = {
    "maze_ood": dict(vocab_size=4, channels=16, c_in=16, c_out=2, output_tokens=(0, 1),
                     perception="kernels", hidden_from_perception=True, heads=4, padding="wall",
                     wall_token=2, update="mlp", expansion=2, norm_groups=0, sigma_init=0.15,
                     fire_rate=0.8, head="l2", embedding="onehot"),
    "maze_hard": dict(vocab_size=5, channels=32, c_in=32, c_out=3, output_tokens=(0, 1),
                      perception="kernels", hidden_from_perception=True, heads=4, padding="wall",
                      wall_token=2, update="mlp", expansion=2, norm_groups=0, sigma_init=0.25,
                      fire_rate=0.8, head="l2", embedding="onehot"),
}


def unsupported_reason(cfg) -> str | None:
    """Why the B200 kernels cannot run this cell rule (None when they can).  Accepts the
    reference's NCAConfig as well as ours."""
    if cfg.perception != "kernels" or cfg.heads != 4:
        return f"perception={cfg.perception!r} heads={cfg.heads} (needs 4-head 'kernels')"
    if cfg.padding not in ("zero", "wall"):
        return f"padding={cfg.padding!r} (needs 'zero' or 'wall')"
    if cfg.update != "mlp":
        return f"update={cfg.update!r} (needs 'mlp')"
    if cfg.norm_groups:
        return "group normalisation"
    if cfg.time_steps or cfg.c_task or cfg.n_tasks:
        return "step or task embeddings"
    if cfg.head not in ("mlp", "l2"):
        return f"head={cfg.head!r} (needs 'mlp' or 'l2')"
    if cfg.embedding != "onehot":
        return f"embedding={cfg.embedding!r} (needs 'onehot')"
    if getattr(cfg, "project_update", False) or getattr(cfg, "noise_after_norm", False):
        return "public-code update switches"
    hid = cfg.expansion * (cfg.heads * cfg.channels if cfg.hidden_from_perception else cfg.channels)
    if (cfg.channels, hid) not in KERNEL_SHAPES:
        return f"channels={cfg.channels}, hidden={hid} (kernels exist for {sorted(KERNEL_SHAPES)})"
    if cfg.c_out > 16 or len(cfg.output_tokens) > 16:
        return "more than 16 readout channels or tokens"
    return None


def check_supported(cfg) -> None:
    why = unsupported_reason(cfg)
    if why is not None:
        raise ValueError(f"the b200 backend does not implement this cell rule: {why}")


def make_embeddings(vocab_size: int, dim: int, kind: str = "onehot") -> torch.Tensor:
    """Fixed token embeddings; `onehot` as src/nca/embeddings.py:38-41."""
    if vocab_size > dim:
        raise ValueError(f"need dim >= vocab_size, got dim={dim} < V={vocab_size}")
    if kind != "onehot":
        raise ValueError(f"embedding {kind!r} is not implemented by the b200 backend")
    return torch.eye(vocab_size, dim)


class KernelPerception(nn.Module):
    def __init__(self, channels: int, heads: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(heads, 1, 3, 3))
        self.channels, self.heads, self.out_dim = channels, heads, heads * channels


class MLPUpdate(nn.Module):
    def __init__(self, in_dim: int, channels: int, hidden: int):
        super().__init__()
        self.fc1 = nn.Conv2d(in_dim, hidden, 1)
        self.fc2 = nn.Conv2d(hidden, channels, 1)


class NCA(nn.Module):
    """Parameter container with the reference's names; compute goes through the B200 engine."""

    def __init__(self, cfg: NCAConfig, precision: str = "bf16"):
        super().__init__()
        self.cfg = cfg
        self.precision = precision
        self.register_buffer("embed", make_embeddings(cfg.vocab_size, cfg.c_in, cfg.embedding))
        # embeddings of the predictable tokens in the output slice (l2 head), and the state of
        # the cells outside the board (wall padding: the wall token's embedding in the input
        # slice), as the reference's buffers (src/nca/model.py:314-325)
        if cfg.head in ("l2", "cosine"):
            lo = cfg.out_offset - cfg.in_offset
            self.register_buffer("out_embed", self.embed[list(cfg.output_tokens)][:, lo : lo + cfg.c_out].clone())
        pad_vec = torch.zeros(cfg.channels)
        if cfg.padding == "wall":
            pad_vec[cfg.in_slice] = self.embed[cfg.wall_token]
        self.register_buffer("pad_vec", pad_vec)
        self.perceive = KernelPerception(cfg.channels, cfg.heads)
        self.update = MLPUpdate(cfg.heads * cfg.channels, cfg.channels, cfg.hidden)
        if cfg.head == "mlp":
            self.head = nn.Conv2d(cfg.c_out, len(cfg.output_tokens), 1)
        self._engine = None

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def engine(self):
        """The B200Engine of this model (weights packed once; call `refresh()` after edits)."""
        from .engine import B200Engine

        if self._engine is None or self._engine.device != self.device:
            self._engine = B200Engine(self, precision=self.precision)
        return self._engine

    def refresh(self) -> None:
        self._engine = None

    # -------------------------------------------------------------- reference API (rollout path)
    def clamp_values(self, inputs: torch.Tensor) -> torch.Tensor:
        return self.embed[inputs].permute(0, 3, 1, 2).contiguous()

    @torch.no_grad()
    def init_state(self, inputs, given, task_ids=None, generator=None):
        """(x, given4, clamp) of a batch (src/nca/model.py:384-412): the state drawn as
        randn * sigma_init (the draw is made so that a shared generator advances exactly as in
        the reference), then the given cells clamped by the library."""
        cfg = self.cfg
        B, H, W = inputs.shape
        x = torch.randn((B, cfg.channels, H, W), generator=generator, device=self.device) * cfg.sigma_init
        given4 = given[:, None].to(self.device)
        clamp = self.clamp_values(inputs.to(self.device))
        return self.apply_clamp(x, given4, clamp), given4, clamp

    @torch.no_grad()
    def apply_clamp(self, x, given4, clamp):
        return self.engine().apply_clamp_nchw(x, given4, clamp)

    @torch.no_grad()
    def step(self, x, given4, clamp, fire_mask, noise=None, clock=None):
        """One asynchronous step (src/nca/model.py:503-525) in the B200 kernel."""
        if noise is not None or clock is not None:
            raise ValueError("the b200 backend has no step noise or clocks")
        return self.engine().step_nchw(x, given4, clamp, fire_mask)

    @torch.no_grad()
    def sample_fire_mask(self, x, p_fire=None, p_low=None, tau=None, generator=None, given=None):
        """Bernoulli firing mask (src/nca/model.py:567-593), uniform rule only."""
        if p_low is not None or tau is not None:
            raise ValueError("threshold adaptive firing is not implemented by the b200 backend")
        p = self.cfg.fire_rate if p_fire is None else p_fire
        B, _, H, W = x.shape
        u = torch.rand((B, 1, H, W), generator=generator, device=x.device)
        return (u < p).to(x.dtype)

    @torch.no_grad()
    def decode(self, x):
        return self.engine().readout_nchw(x)["decoded"]

    @torch.no_grad()
    def confidence(self, x):
        return self.engine().readout_nchw(x)["cell_conf"]

    @torch.no_grad()
    def board_confidence(self, x):
        return self.engine().readout_nchw(x)["board_conf"]


def build_model(preset: str | None = None, precision: str = "bf16", **overrides) -> NCA:
    """`build_model("maze_hard")` or `build_model(None, **cfg_fields)` as src/nca/model.py:766-771;
    the presets whose cell rule the kernels implement are in PRESETS."""
    if preset is not None and preset not in PRESETS:
        raise ValueError(f"preset {preset!r} needs a cell rule the b200 kernels do not implement "
                         f"(available: {sorted(PRESETS)})")
    d = dict(PRESETS[preset]) if preset else {}
    d.update(overrides)
    d["output_tokens"] = tuple(d["output_tokens"])
    return NCA(NCAConfig(**d), precision=precision)


def load_model(path, device=None, precision: str = "bf16"):
    """A trained checkpoint (the reference's final.pt: model_config, EMA weights, run config) as
    nca.train.load_model (src/nca/train.py:694-701): returns (model, run config)."""
    ck = torch.load(path, map_location="cpu", weights_only=False)
    model = NCA(NCAConfig.from_dict(dict(ck["model_config"])), precision=precision)
    model.load_state_dict(ck["model"])
    if device is not None:
        model = model.to(device)
    return model.eval(), ck.get("config", {})
