"""The five decode configurations of the north-star spec and device-side
synthetic inputs for them.

Inputs are seeded N(0,1) fp32 for Q and for the K/V rows, which are quantised
per token on the GPU by the library's own quantiser (kvd_quantize_rows_launch,
bit-exact with the host spec). No dataset is involved: the reference measures
nothing on public data for this path, so seeded synthetic data of the stated
shapes stands in.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import kvdecode as kvd


@dataclass
class Config:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    head_dim: int
    seq_len: int                 # dense length, or the capacity for ragged batches
    ragged: tuple | None = None  # (lo, hi) inclusive range of per-sequence lengths
    append: bool = False
    notes: str = ""

    @property
    def group(self) -> int:
        return self.q_heads // self.kv_heads


CONFIGS = {
    1: Config("mha_small", 1, 8, 8, 64, 1024, notes="CPU-checkable MHA"),
    2: Config("llama7b_mha", 64, 32, 32, 128, 4096, notes="Llama-7B-like MHA"),
    3: Config("long_context", 4, 32, 32, 128, 131072, notes="long-context MHA"),
    4: Config("ragged_append", 128, 32, 32, 128, 8193, ragged=(256, 8192), append=True,
              notes="ragged batch with quantise-on-append of one token"),
    5: Config("gqa8", 256, 64, 8, 128, 2048, notes="GQA, group 8"),
}


def ragged_lengths(cfg: Config, seed: int):
    """Per-sequence lengths drawn uniformly in [lo, hi] from the seed (host list)."""
    import numpy as np

    lo, hi = cfg.ragged
    return np.random.default_rng(seed).integers(lo, hi + 1, size=cfg.batch).astype("int32").tolist()


@dataclass
class DeviceCase:
    cfg: Config
    q: object
    K: object
    V: object
    ks: object
    vs: object
    seq_lens: object = None          # device int32 [B] (ragged)
    lens_host: list = field(default_factory=list)
    k_new: object = None             # fp32 [B, Hkv, D] token to append (ragged config)
    v_new: object = None


def fill_quantised(codes, scales, gen, chunk_rows: int = 1 << 22) -> None:
    """Fill a [..., D] int8 cache and its [...] scales with quantised N(0,1) rows."""
    import torch

    D = codes.shape[-1]
    c2 = codes.view(-1, D)
    s1 = scales.view(-1)
    rows = c2.shape[0]
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        x = torch.randn((r1 - r0, D), generator=gen, device=codes.device, dtype=torch.float32)
        kvd.quantize_rows(x, c2[r0:r1], s1[r0:r1])
        del x


def make_case(cfg: Config, seed: int = 17, device: str = "cuda", batch: int | None = None) -> DeviceCase:
    """Allocates and fills one configuration on the device (`batch` overrides cfg.batch)."""
    import torch

    B = cfg.batch if batch is None else batch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    q = torch.randn((B, cfg.q_heads, cfg.head_dim), generator=gen, device=device, dtype=torch.float32)
    shape = (B, cfg.kv_heads, cfg.seq_len, cfg.head_dim)
    K = torch.empty(shape, dtype=torch.int8, device=device)
    V = torch.empty(shape, dtype=torch.int8, device=device)
    ks = torch.empty(shape[:3], dtype=torch.float32, device=device)
    vs = torch.empty(shape[:3], dtype=torch.float32, device=device)
    fill_quantised(K, ks, gen)
    fill_quantised(V, vs, gen)
    case = DeviceCase(cfg, q, K, V, ks, vs)
    if cfg.ragged:
        lens = ragged_lengths(cfg, seed)[:B]
        case.lens_host = lens
        case.seq_lens = torch.tensor(lens, dtype=torch.int32, device=device)
        case.k_new = torch.randn((B, cfg.kv_heads, cfg.head_dim), generator=gen, device=device)
        case.v_new = torch.randn((B, cfg.kv_heads, cfg.head_dim), generator=gen, device=device)
    torch.cuda.synchronize()
    return case


def parity_items(cfg: Config, batch: int, lens=None, min_rows: int = 64, seed: int = 5) -> list:
    """(b, kv head) items whose query rows a full-size parity check compares:
    at least `min_rows` query rows, always the first and last sequence, the last
    kv head and, for ragged batches, the longest and shortest sequence; the rest
    drawn from the seed. Each item covers the group's Hq/Hkv query heads."""
    import numpy as np

    B, Hkv, G = batch, cfg.kv_heads, cfg.group
    want = max(1, -(-min_rows // G))
    items = [(0, 0), (B - 1, Hkv - 1), (0, Hkv - 1), (B - 1, 0)]
    if lens is not None and len(lens):
        lens = list(lens)
        items += [(int(np.argmax(lens)), Hkv // 2), (int(np.argmin(lens)), Hkv - 1)]
    rng = np.random.default_rng(seed)
    while len(set(items)) < min(want, B * Hkv):
        items.append((int(rng.integers(B)), int(rng.integers(Hkv))))
    out, seen = [], set()
    for it in items:
        if it not in seen:
            seen.add(it)
            out.append(it)
    return out


def step_bytes(cfg: Config, lens=None, batch: int | None = None) -> int:
    """Algorithmic HBM bytes of one decode step (plus append traffic when it runs)."""
    B = cfg.batch if batch is None else batch
    if cfg.ragged:
        total = kvd.algorithmic_bytes(B, cfg.q_heads, cfg.kv_heads, cfg.head_dim, lens)
        if cfg.append:  # read 2 fp32 rows, write 2 code rows + 2 scales per (b, kv head)
            total += B * cfg.kv_heads * (2 * cfg.head_dim * 4 + 2 * (cfg.head_dim + 4))
        return total
    return kvd.algorithmic_bytes(B, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.seq_len)
