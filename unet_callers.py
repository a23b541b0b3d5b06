"""UNet callers of the NOVA 3x3 path: the SD 1.5 and SDXL UNet layouts.

Benchmark callers for configs 4 and 5 (one denoising step of a random-init
UNet with every eligible 3x3 stride-1 conv on NOVA F(6,3)).  ``diffusers`` is
not installed, so the two layouts are restated here from their published
shapes:

- SD 1.5: levels of 320 / 640 / 1280 / 1280 channels, 2 residual blocks per
  level going down and 3 coming up, one cross-attention transformer layer on
  the first three levels and in the middle, 8 heads, 768-wide text context,
  1x1-conv projections around each transformer.  49 eligible 3x3 stride-1
  convs.
- SDXL: levels of 320 / 640 / 1280 channels, no attention on the first level,
  2 and 10 transformer layers on the next two and 10 in the middle, 64-wide
  heads, 2048-wide context, linear projections, and an added embedding of
  the pooled text vector (1280) and six time ids.  38 eligible convs.

Both use GroupNorm(32) + SiLU residual blocks with the time embedding added
between the two 3x3 convs, stride-2 3x3 downsampling convs (not eligible) and
nearest-neighbour x2 upsampling followed by a 3x3 stride-1 conv (eligible).
"""

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class UNetSpec:
    channels: tuple           # per level, top (full resolution) first
    attn_depth: tuple         # transformer layers per level (0 = none)
    mid_depth: int            # transformer layers in the middle block
    context_dim: int
    heads: int = 0            # fixed head count (SD 1.5), or
    head_dim: int = 0         # fixed head width (SDXL)
    linear_proj: bool = False  # linear (SDXL) or 1x1-conv (SD 1.5) transformer projections
    add_embed: bool = False   # SDXL pooled-text + time-id embedding
    layers_per_level: int = 2
    in_ch: int = 4
    out_ch: int = 4
    groups: int = 32
    time_freq_dim: int = 0    # sinusoid width of the timestep; 0 = channels[0]
    add_time_dim: int = 256   # sinusoid width per SDXL time id
    pooled_dim: int = 1280
    n_time_ids: int = 6


SD15 = UNetSpec(channels=(320, 640, 1280, 1280), attn_depth=(1, 1, 1, 0), mid_depth=1,
                context_dim=768, heads=8)
SDXL = UNetSpec(channels=(320, 640, 1280), attn_depth=(0, 2, 10), mid_depth=10,
                context_dim=2048, head_dim=64, linear_proj=True, add_embed=True)


def sinusoid(t, dim):
    """Sinusoidal embedding of a float tensor t (any shape) -> [..., dim]:
    cos terms first, then sin, frequencies 10000^(-i / (dim/2))."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device,
                                                         dtype=torch.float32) / half)
    ang = t.float()[..., None] * freqs
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1)


class ResBlock(nn.Module):
    def __init__(self, cin, cout, temb_dim, groups):
        super().__init__()
        self.norm1 = nn.GroupNorm(groups, cin, eps=1e-5)
        self.conv1 = nn.Conv2d(cin, cout, 3, padding=1)
        self.temb = nn.Linear(temb_dim, cout)
        self.norm2 = nn.GroupNorm(groups, cout, eps=1e-5)
        self.conv2 = nn.Conv2d(cout, cout, 3, padding=1)
        self.skip = nn.Conv2d(cin, cout, 1) if cin != cout else nn.Identity()

    def forward(self, x, temb):
        h = self.conv1(F.silu(self.norm1(x)))
        h = h + self.temb(F.silu(temb))[:, :, None, None]
        h = self.conv2(F.silu(self.norm2(h)))
        return self.skip(x) + h


class Attention(nn.Module):
    def __init__(self, dim, ctx_dim, heads):
        super().__init__()
        self.heads = heads
        self.q = nn.Linear(dim, dim, bias=False)
        self.k = nn.Linear(ctx_dim, dim, bias=False)
        self.v = nn.Linear(ctx_dim, dim, bias=False)
        self.out = nn.Linear(dim, dim)

    def forward(self, x, ctx=None):
        ctx = x if ctx is None else ctx
        B, N, D = x.shape
        h = self.heads

        def split(t):
            return t.view(B, -1, h, D // h).transpose(1, 2)

        o = F.scaled_dot_product_attention(split(self.q(x)), split(self.k(ctx)), split(self.v(ctx)))
        return self.out(o.transpose(1, 2).reshape(B, N, D))


class TransformerLayer(nn.Module):
    def __init__(self, dim, ctx_dim, heads):
        super().__init__()
        self.n1, self.self_attn = nn.LayerNorm(dim), Attention(dim, dim, heads)
        self.n2, self.cross_attn = nn.LayerNorm(dim), Attention(dim, ctx_dim, heads)
        self.n3 = nn.LayerNorm(dim)
        self.ff_in = nn.Linear(dim, 8 * dim)   # GEGLU: value and gate halves
        self.ff_out = nn.Linear(4 * dim, dim)

    def forward(self, x, ctx):
        x = x + self.self_attn(self.n1(x))
        x = x + self.cross_attn(self.n2(x), ctx)
        a, g = self.ff_in(self.n3(x)).chunk(2, dim=-1)
        return x + self.ff_out(a * F.gelu(g))


class Transformer2D(nn.Module):
    def __init__(self, ch, depth, spec):
        super().__init__()
        heads = spec.heads if spec.heads else ch // spec.head_dim
        self.linear = spec.linear_proj
        self.norm = nn.GroupNorm(spec.groups, ch, eps=1e-6)
        self.proj_in = nn.Linear(ch, ch) if self.linear else nn.Conv2d(ch, ch, 1)
        self.layers = nn.ModuleList(TransformerLayer(ch, spec.context_dim, heads)
                                    for _ in range(depth))
        self.proj_out = nn.Linear(ch, ch) if self.linear else nn.Conv2d(ch, ch, 1)

    def forward(self, x, ctx):
        B, C, H, W = x.shape
        h = self.norm(x)
        if self.linear:
            h = self.proj_in(h.flatten(2).transpose(1, 2))
        else:
            h = self.proj_in(h).flatten(2).transpose(1, 2)
        for layer in self.layers:
            h = layer(h, ctx)
        if self.linear:
            h = self.proj_out(h).transpose(1, 2).reshape(B, C, H, W)
        else:
            h = self.proj_out(h.transpose(1, 2).reshape(B, C, H, W))
        return x + h


class Level(nn.Module):
    """Residual blocks of one level, each optionally followed by a transformer."""

    def __init__(self, cins, cout, depth, temb_dim, spec):
        super().__init__()
        self.res = nn.ModuleList(ResBlock(c, cout, temb_dim, spec.groups) for c in cins)
        self.attn = nn.ModuleList(Transformer2D(cout, depth, spec) for _ in cins) if depth else None


class UNet(nn.Module):
    def __init__(self, spec: UNetSpec):
        super().__init__()
        self.spec = spec
        ch = spec.channels
        self.freq_dim = spec.time_freq_dim or ch[0]
        temb = 4 * ch[0]
        self.time_mlp = nn.Sequential(nn.Linear(self.freq_dim, temb), nn.SiLU(),
                                      nn.Linear(temb, temb))
        if spec.add_embed:
            add_in = spec.pooled_dim + spec.n_time_ids * spec.add_time_dim
            self.add_mlp = nn.Sequential(nn.Linear(add_in, temb), nn.SiLU(), nn.Linear(temb, temb))
        self.conv_in = nn.Conv2d(spec.in_ch, ch[0], 3, padding=1)

        skips = [ch[0]]
        self.down = nn.ModuleList()
        self.downsample = nn.ModuleList()
        cur = ch[0]
        for i, c in enumerate(ch):
            cins = [cur] + [c] * (spec.layers_per_level - 1)
            self.down.append(Level(cins, c, spec.attn_depth[i], temb, spec))
            cur = c
            skips += [c] * spec.layers_per_level
            if i < len(ch) - 1:
                self.downsample.append(nn.Conv2d(c, c, 3, stride=2, padding=1))
                skips.append(c)

        self.mid_res1 = ResBlock(cur, cur, temb, spec.groups)
        self.mid_attn = Transformer2D(cur, spec.mid_depth, spec)
        self.mid_res2 = ResBlock(cur, cur, temb, spec.groups)

        self.up = nn.ModuleList()
        self.upsample = nn.ModuleList()
        for i, c in reversed(list(enumerate(ch))):
            cins = []
            for _ in range(spec.layers_per_level + 1):
                cins.append(cur + skips.pop())
                cur = c
            self.up.append(Level(cins, c, spec.attn_depth[i], temb, spec))
            if i > 0:
                self.upsample.append(nn.Conv2d(c, c, 3, padding=1))
        assert not skips
        self.norm_out = nn.GroupNorm(spec.groups, ch[0], eps=1e-5)
        self.conv_out = nn.Conv2d(ch[0], spec.out_ch, 3, padding=1)

    def forward(self, x, t, ctx, pooled=None, time_ids=None):
        """x: [B, 4, h, w] latent; t: [B] timesteps; ctx: [B, 77, context_dim];
        SDXL also pooled [B, 1280] and time_ids [B, 6]."""
        dt = x.dtype
        temb = self.time_mlp(sinusoid(t, self.freq_dim).to(dt))
        if self.spec.add_embed:
            ids = sinusoid(time_ids, self.spec.add_time_dim).flatten(1).to(dt)
            temb = temb + self.add_mlp(torch.cat([pooled.to(dt), ids], dim=1))
        h = self.conv_in(x)
        hs = [h]
        for i, lvl in enumerate(self.down):
            for j, rb in enumerate(lvl.res):
                h = rb(h, temb)
                if lvl.attn is not None:
                    h = lvl.attn[j](h, ctx)
                hs.append(h)
            if i < len(self.downsample):
                h = self.downsample[i](h)
                hs.append(h)
        h = self.mid_res2(self.mid_attn(self.mid_res1(h, temb), ctx), temb)
        for i, lvl in enumerate(self.up):
            for j, rb in enumerate(lvl.res):
                h = rb(torch.cat([h, hs.pop()], dim=1), temb)
                if lvl.attn is not None:
                    h = lvl.attn[j](h, ctx)
            if i < len(self.upsample):
                h = self.upsample[i](F.interpolate(h, scale_factor=2.0, mode="nearest"))
        return self.conv_out(F.silu(self.norm_out(h)))


def make_inputs(spec, batch, latent, device, dtype=torch.float16, seed=0):
    """Synthetic step inputs of the config: N(0,1) latent and context, integer
    timesteps in [0, 1000); for SDXL N(0,1) pooled text and six time ids
    (original size, crop offset, target size)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(batch, spec.in_ch, latent, latent, generator=g).to(device, dtype)
    t = torch.randint(0, 1000, (batch,), generator=g).to(device)
    ctx = torch.randn(batch, 77, spec.context_dim, generator=g).to(device, dtype)
    extra = {}
    if spec.add_embed:
        extra["pooled"] = torch.randn(batch, spec.pooled_dim, generator=g).to(device, dtype)
        side = float(latent * 8)
        extra["time_ids"] = torch.tensor([[side, side, 0.0, 0.0, side, side]] * batch,
                                         device=device)
    return x, t, ctx, extra
