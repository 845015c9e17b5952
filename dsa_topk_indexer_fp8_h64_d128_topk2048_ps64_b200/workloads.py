"""Seeded synthetic inputs for the indexer (the contest workloads are not
available, so these stand in for them with the shapes and value
distributions of the five benchmark configurations).

Distributions: q ~ N(0,1) cast to e4m3; every cached token k ~ N(0,1)^128 is
quantised per token with scale = amax/448 to e4m3 and packed into the 8448-B
page layout (64x128 e4m3 values, then 64 fp32 scales); weights ~ N(0,1)/8;
the block table maps each row's logical pages onto a seeded random
permutation of the physical pool.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import HEAD_DIM, NUM_HEADS, PAGE_BYTES, PAGE_SIZE, SCALE_OFFSET, TOPK

FP8 = torch.float8_e4m3fn


@dataclass
class Inputs:
    q: torch.Tensor            # [rows, 64, 128] float8_e4m3fn
    k_cache: torch.Tensor      # [num_pages, 64, 1, 132] uint8
    weights: torch.Tensor      # [rows, 64] fp32
    seq_lens: torch.Tensor     # [rows] int32
    block_table: torch.Tensor  # [rows, max_pages] int32
    name: str = ""
    seed: int = 0
    planted: dict = field(default_factory=dict)  # row -> list of planted token indices
    rows_per_seq: int = 1      # consecutive rows sharing one sequence's block-table row

    @property
    def rows(self) -> int:
        return int(self.block_table.shape[0])

    @property
    def max_pages(self) -> int:
        return int(self.block_table.shape[1])

    @property
    def num_pages(self) -> int:
        return int(self.k_cache.shape[0])

    def out(self) -> torch.Tensor:
        return torch.full((self.rows, TOPK), -7, dtype=torch.int32, device=self.block_table.device)

    def to(self, device) -> "Inputs":
        return Inputs(self.q.to(device), self.k_cache.to(device), self.weights.to(device),
                      self.seq_lens.to(device), self.block_table.to(device), self.name, self.seed,
                      dict(self.planted), self.rows_per_seq)

    def numpy(self) -> dict:
        """Host copies for the CPU oracle (q and k as raw bytes)."""
        return dict(q=self.q.view(torch.uint8).cpu().numpy(),
                    k_cache=self.k_cache.cpu().numpy(),
                    weights=self.weights.cpu().numpy(),
                    seq_lens=self.seq_lens.cpu().numpy(),
                    block_table=self.block_table.cpu().numpy(),
                    num_pages=self.num_pages)

    def algorithmic_bytes(self) -> int:
        """Bytes the operator must move per call: per scored row 132*L of
        index-K + 4*ceil(L/64) of block table + 8192 (q) + 256 (weights) + 4
        (seq_len) + 8192 (output); rows with L <= 2048 move only the block
        table, seq_len and output.  With rows_per_seq > 1 a group of rows
        that shares a sequence reads its index-K and block table once, for
        its longest row (132*Lmax + 4*ceil(Lmax/64)), when any of its rows is
        scored; q, weights, seq_len and output stay per row.  Logit scratch is
        not counted."""
        sl = self.seq_lens.cpu().numpy().astype(np.int64)
        sl = np.clip(sl, 0, self.max_pages * PAGE_SIZE)
        pages = (sl + PAGE_SIZE - 1) // PAGE_SIZE
        scored = sl > TOPK
        R = max(1, self.rows_per_seq)
        if R == 1:
            per = np.where(scored, 132 * sl + 8192 + 256, 0) + 4 * pages + 4 + 4 * TOPK
            return int(per.sum())
        lmax = sl.reshape(-1, R).max(axis=1)
        g_scored = lmax > TOPK
        shared = np.where(g_scored, 132 * lmax, 0) + 4 * ((lmax + PAGE_SIZE - 1) // PAGE_SIZE)
        per_row = np.where(np.repeat(g_scored, R), 8192 + 256, 0) + 4 + 4 * TOPK
        return int(shared.sum() + per_row.sum())

    def subset(self, rows, device="cpu") -> "Inputs":
        """The batch restricted to `rows`, with only the pages those rows
        reach, copied into a compact pool (block-table entries remapped,
        entries past a row's last page set to 0).  Gives a small host copy
        of a few rows of a batch whose full pool is too large to copy."""
        rows = [int(r) for r in rows]
        sl = self.seq_lens.cpu()[rows].to(torch.int64).clamp(0, self.max_pages * PAGE_SIZE)
        bt = self.block_table.cpu()[rows].to(torch.int64)
        npg = ((sl + PAGE_SIZE - 1) // PAGE_SIZE).tolist()
        used = torch.unique(torch.cat([bt[i, :n] for i, n in enumerate(npg)] + [torch.zeros(1, dtype=torch.int64)]))
        remap = {int(p): i for i, p in enumerate(used.tolist())}
        bt_new = torch.zeros_like(bt)
        for i, n in enumerate(npg):
            bt_new[i, :n] = torch.tensor([remap[int(p)] for p in bt[i, :n].tolist()], dtype=torch.int64)
        k_new = self.k_cache[used.to(self.k_cache.device)].to(device)
        return Inputs(self.q[rows].to(device), k_new, self.weights[rows].to(device),
                      sl.to(torch.int32).to(device), bt_new.to(torch.int32).to(device),
                      name=f"{self.name}[{len(rows)} rows]", seed=self.seed, rows_per_seq=1)

    def scored_tokens(self) -> int:
        sl = self.seq_lens.cpu().numpy().astype(np.int64)
        sl = np.clip(sl, 0, self.max_pages * PAGE_SIZE)
        return int(sl[sl > TOPK].sum())


def quantize_tokens(k: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token e4m3 quantisation: scale = amax/448, values k/scale."""
    amax = k.abs().amax(dim=-1, keepdim=True).clamp_min(1e-12)
    scale = (amax / 448.0).to(torch.float32)
    kq = (k / scale).clamp(-448.0, 448.0).to(FP8)
    return kq, scale.squeeze(-1)


def pack_pages(kq: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """[n_pages*64, 128] e4m3 + [n_pages*64] fp32 -> [n_pages, 64, 1, 132] u8
    in the split page layout (K block first, scales at byte 8192)."""
    n_pages = kq.shape[0] // PAGE_SIZE
    out = torch.empty((n_pages, PAGE_BYTES), dtype=torch.uint8, device=kq.device)
    out[:, :SCALE_OFFSET] = kq.view(torch.uint8).reshape(n_pages, SCALE_OFFSET)
    out[:, SCALE_OFFSET:] = scale.reshape(n_pages, PAGE_SIZE).contiguous().view(torch.uint8).reshape(
        n_pages, PAGE_SIZE * 4)
    return out.view(n_pages, PAGE_SIZE, 1, 132)


def unpack_pages(k_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of pack_pages: ([n_pages, 64, 128] e4m3, [n_pages, 64] fp32)."""
    flat = k_cache.reshape(-1, PAGE_BYTES)
    kq = flat[:, :SCALE_OFFSET].contiguous().view(FP8).reshape(-1, PAGE_SIZE, HEAD_DIM)
    sc = flat[:, SCALE_OFFSET:].contiguous().view(torch.float32).reshape(-1, PAGE_SIZE)
    return kq, sc


def make_inputs(seq_lens, *, max_pages: int | None = None, pool_pages: int | None = None,
                slack: float = 1.1, seed: int = 0, device="cpu", name: str = "",
                share_rows: int = 1, chunk_pages: int = 4096) -> Inputs:
    """Builds one batch.  `share_rows` > 1 makes consecutive groups of that
    many rows share one block-table row (multi-query: several query rows of
    one sequence); the group's pages cover its longest row."""
    device = torch.device(device)
    sl = np.asarray(seq_lens, dtype=np.int64)
    rows = int(sl.shape[0])
    rng = np.random.RandomState(seed)
    pages_per_row = (sl + PAGE_SIZE - 1) // PAGE_SIZE
    groups = rows // share_rows
    gpages = [int(pages_per_row[g * share_rows:(g + 1) * share_rows].max()) for g in range(groups)]
    need = int(sum(gpages))
    if max_pages is None:
        max_pages = max(1, int(pages_per_row.max()) if rows else 1)
    if pool_pages is None:
        pool_pages = max(1, int(math.ceil(need * slack)))
    assert pool_pages >= need, "pool too small"
    perm = rng.permutation(pool_pages).astype(np.int32)
    bt = np.zeros((rows, max_pages), dtype=np.int32)
    pos = 0
    for g in range(groups):
        ids = perm[pos:pos + gpages[g]]
        pos += gpages[g]
        for r in range(g * share_rows, (g + 1) * share_rows):
            bt[r, :gpages[g]] = ids

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    q = torch.randn((rows, NUM_HEADS, HEAD_DIM), generator=gen, device=device).to(FP8)
    weights = (torch.randn((rows, NUM_HEADS), generator=gen, device=device) / 8.0).to(torch.float32)
    k_cache = torch.empty((pool_pages, PAGE_SIZE, 1, 132), dtype=torch.uint8, device=device)
    for p0 in range(0, pool_pages, chunk_pages):
        p1 = min(pool_pages, p0 + chunk_pages)
        k = torch.randn(((p1 - p0) * PAGE_SIZE, HEAD_DIM), generator=gen, device=device)
        kq, sc = quantize_tokens(k)
        k_cache[p0:p1] = pack_pages(kq, sc)
    return Inputs(q, k_cache, weights.contiguous(),
                  torch.from_numpy(sl.astype(np.int32)).to(device),
                  torch.from_numpy(bt).to(device), name=name, seed=seed, rows_per_seq=share_rows)


def plant_tokens(inp: Inputs, row: int, tokens, boost: float = 4.0) -> None:
    """Overwrites the K of `tokens` of `row` with a vector aligned to the
    row's positively weighted query heads, so their logits are far above the
    rest (used to check that a split row's merge keeps them)."""
    qd = inp.q[row].to(torch.float32)                      # [64, 128]
    w = inp.weights[row].clamp_min(0.0)                    # [64]
    direction = (w[:, None] * qd).sum(0)
    direction = direction / direction.norm().clamp_min(1e-6) * math.sqrt(HEAD_DIM) * boost
    kq, sc = quantize_tokens(direction[None, :].expand(len(tokens), HEAD_DIM).contiguous())
    flat = inp.k_cache.view(-1, PAGE_BYTES)
    bt = inp.block_table[row].cpu().numpy()
    for i, t in enumerate(tokens):
        page, slot = int(bt[t // PAGE_SIZE]), t % PAGE_SIZE
        flat[page, slot * HEAD_DIM:(slot + 1) * HEAD_DIM] = kq[i].view(torch.uint8)
        flat[page, SCALE_OFFSET + 4 * slot:SCALE_OFFSET + 4 * slot + 4] = sc[i:i + 1].view(torch.uint8)
    inp.planted.setdefault(row, []).extend(int(t) for t in tokens)


def _uniform_lengths(rng: np.random.RandomState, n: int, lo: int, hi: int) -> np.ndarray:
    sl = rng.randint(lo, hi + 1, size=n)
    sl = np.where(sl % PAGE_SIZE == 0, sl - 1, sl)  # not page multiples
    return sl


CONFIGS = {
    0: "decode B=2, seq_lens {1500, 4096}, 88-page pool (CPU-runnable case)",
    1: "decode B=64, seq_lens U[4096, 32768]",
    2: "decode B=256, seq_lens U[65536, 131072] (rows split across GPUs)",
    3: "single request B=1, seq_len 131072, 16 planted tokens (page-range split)",
    4: "multi-query 32 seqs x 4 rows, causal seq_lens L-3..L, L U[8192, 65536]",
}


def prefill_inputs(chunk: int, last_len: int, *, seed: int = 7, device="cpu", rows_per_seq: int = 4) -> Inputs:
    """The indexer rows of one prefill chunk: `chunk` query tokens of one
    sequence at positions last_len - chunk .. last_len - 1, so row i sees the
    causal prefix of length last_len - chunk + 1 + i; every row holds the
    sequence's block-table row.  The kernel scores them in groups of
    `rows_per_seq` consecutive rows (each group reads the K pages once)."""
    sl = np.arange(last_len - chunk + 1, last_len + 1)
    inp = make_inputs(sl, seed=seed, device=device, name=f"prefill{chunk}x{last_len}", share_rows=chunk)
    inp.rows_per_seq = rows_per_seq
    return inp


def config_inputs(config: int, *, seed: int | None = None, device="cpu", rows: int | None = None) -> Inputs:
    """Inputs of one benchmark configuration (`rows` shrinks the batch for a
    quick case of the same distribution)."""
    seed = config if seed is None else seed
    rng = np.random.RandomState(1000 + seed)
    if config == 0:
        return make_inputs([1500, 4096], max_pages=64, pool_pages=88, seed=seed, device=device,
                           name="config0")
    if config == 1:
        n = rows or 64
        return make_inputs(_uniform_lengths(rng, n, 4096, 32768), seed=seed, device=device, name="config1")
    if config == 2:
        n = rows or 256
        return make_inputs(_uniform_lengths(rng, n, 65536, 131072), seed=seed, device=device, name="config2")
    if config == 3:
        inp = make_inputs([131072], seed=seed, device=device, name="config3")
        L = 131072
        # 16 planted tokens, half of them next to the 2/4/8-way page-range cuts
        cuts = sorted({L * i // g for g in (2, 4, 8) for i in range(1, g)})
        chosen = {c + int(rng.randint(-3, 3)) for c in cuts[:8]}
        while len(chosen) < 16:
            chosen.add(int(rng.randint(0, L)))
        plant_tokens(inp, 0, sorted(chosen))
        return inp
    if config == 4:
        n_seq = (rows // 4) if rows else 32
        base = rng.randint(8192, 65536 + 1, size=n_seq)
        sl = np.stack([base - 3, base - 2, base - 1, base], axis=1).reshape(-1)
        return make_inputs(sl, seed=seed, device=device, name="config4", share_rows=4)
    raise ValueError(f"unknown config {config}")
