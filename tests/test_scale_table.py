"""The GEMV's per-tile scale table (weights.scale_table), on the CPU: every local row of every rank's shard
(GDN / attention head slices, gate|up interleaved pairs, vocab slices at n = 1, 2, 4, 8) reads, through its
tile's row selector, exactly the canonical fp32 scale of its 128-row block at every K block; unused slots
hold 0; more than 8 blocks in one tile is refused."""
import pytest
import torch

from tt_qwen_resident_b200 import weights


def _decode(tab, nkb):
    tiles = tab.shape[0]
    sel = tab[:, :128].long()
    sc = tab[:, 128:].contiguous().view(torch.float32).view(tiles, nkb, 8)
    return sel, sc


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_scale_table_every_shard_row(n):
    g = torch.Generator().manual_seed(n)
    scales = torch.rand(2000, 40, generator=g) + 0.5
    for r in range(n):
        d = weights.RankDims(r, n, vocab=248320)
        for rows in (d.gdn_rows(), d.attn_rows(), d.gateup_rows(), d.vocab_rows()):
            tab = weights.scale_table(rows // 128, scales, 3, 40)
            sel, sc = _decode(tab, 37)
            tiles = tab.shape[0]
            assert tiles == -(-len(rows) // 128)
            local = torch.arange(tiles * 128).clamp(max=len(rows) - 1)
            got = sc[torch.arange(tiles * 128) // 128, :, sel.reshape(-1)]  # [rows_pad, nkb]
            want = scales[rows[local] // 128][:, 3:40]
            assert torch.equal(got, want)
            used = torch.zeros(tiles, 8, dtype=torch.bool)
            used.scatter_(1, sel, True)
            assert bool((sc.permute(0, 2, 1)[~used] == 0).all())


def test_scale_table_refuses_nine_blocks():
    rows = torch.arange(9).repeat_interleave(14) * 128  # 126 rows from 9 distinct blocks in one tile
    with pytest.raises(ValueError):
        weights.scale_table(rows // 128, torch.ones(9, 2), 0, 2)
