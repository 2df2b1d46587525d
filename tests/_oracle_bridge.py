"""Run the CPU oracle on (a subset of) a device batch.

The device cache can be tens of GB; the oracle gets a compact copy holding
only the pages of the chosen requests, renumbered, taken BEFORE the
operator writes the step's K/V (the oracle writes them itself).
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import OracleMetadata, paged_attention


def snapshot_pages(cache: torch.Tensor, table: torch.Tensor, ctx_lens: list[int], rows: list[int]):
    bs = cache.shape[2]
    pages = []
    for r in rows:
        n = -(-ctx_lens[r] // bs)
        pages.append(table[r, :n].cpu())
    ids = torch.cat(pages) if pages else torch.zeros(0, dtype=torch.int64)
    return cache[:, ids.to(cache.device)].float().cpu().numpy(), pages


def oracle_subset(batch, rows: list[int], snapshot) -> tuple[np.ndarray, list[int]]:
    """Oracle outputs (fp32) for the tokens of `rows`; returns (out, token ids)."""

    compact, pages = snapshot
    md = batch.metadata
    qsl = md.query_start_locations.cpu().numpy()
    pos = md.query_positions.cpu().numpy()
    starts = md.query_context_start_positions.cpu().numpy()
    bs = md.block_size
    tok, new_qsl, new_tables, new_slots, new_pos, new_starts, ctx = [], [0], [], [], [], [], []
    base = 0
    width = max(len(p) for p in pages)
    for r, pg in zip(rows, pages):
        t0, t1 = int(qsl[r]), int(qsl[r + 1])
        tok.extend(range(t0, t1))
        new_qsl.append(new_qsl[-1] + (t1 - t0))
        row = np.arange(base, base + len(pg), dtype=np.int64)
        new_tables.append(np.pad(row, (0, width - len(pg))))
        for t in range(t0, t1):
            p = int(pos[t])
            new_slots.append(row[p // bs] * bs + p % bs)
            new_pos.append(p)
            new_starts.append(int(starts[t]))
        ctx.append(int(batch.context_lengths[r]))
        base += len(pg)
    omd = OracleMetadata(
        query_positions=np.asarray(new_pos, np.int64),
        query_context_start_positions=np.asarray(new_starts, np.int64),
        query_start_locations=np.asarray(new_qsl, np.int64),
        context_lengths=np.asarray(ctx, np.int64),
        block_table=np.stack(new_tables),
        slot_mapping=np.asarray(new_slots, np.int64),
        block_size=bs,
    )
    idx = torch.tensor(tok, dtype=torch.int64)
    q = batch.query.cpu()[idx].float().numpy()
    k = batch.key.cpu()[idx].float().numpy()
    v = batch.value.cpu()[idx].float().numpy()
    out = paged_attention(q, k, v, compact.copy(), omd, out_dtype=np.float32)
    return out, tok


def assert_close(actual: torch.Tensor, expected: np.ndarray, atol: float, rtol: float) -> None:
    a = actual.float().cpu().numpy()
    np.testing.assert_allclose(a, expected, atol=atol, rtol=rtol, equal_nan=True)
