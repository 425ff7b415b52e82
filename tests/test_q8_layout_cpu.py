"""Host repacking of Q8_0 matrices for b2a_q8_gemv (decode_chain.Q8Matrix):
the fragment-order tiles, the scale order, row padding and the 8-row
gate/up interleave, checked element by element on CPU tensors."""
import torch

from alpacca_open_sourced_by_jt_b200.decode_chain import Q8Matrix


def test_tile_fragment_order_and_padding():
    g = torch.Generator().manual_seed(0)
    R, C = 35, 96
    codes = torch.randint(-128, 128, (R, C), dtype=torch.int8, generator=g)
    scales = torch.randn(R, C // 32, generator=g).to(torch.float16)
    tiles, ts = Q8Matrix(codes, scales).tiles()
    assert tiles.shape == (3, 3, 512) and ts.shape == (3, 3, 16)
    for rg in range(3):
        for b in range(3):
            for lane in range(32):
                gg, q = lane // 4, lane % 4
                for j in range(16):
                    m, reg, half = j // 8, (j % 8) // 2, j % 2
                    row = rg * 16 + gg + (8 if reg in (1, 3) else 0)
                    k = b * 32 + 16 * m + 2 * q + half + (8 if reg in (2, 3) else 0)
                    want = codes[row, k] if row < R else 0
                    assert tiles[rg, b, lane * 16 + j] == want
            for i in range(16):
                row = rg * 16 + (i // 2) + (8 if i % 2 else 0)
                want = scales[row, b] if row < R else 0
                assert ts[rg, b, i] == want


def test_gate_up_interleave_by_eight_rows():
    a = Q8Matrix((torch.arange(16 * 32) % 100).to(torch.int8).view(16, 32),
                 torch.ones(16, 1, dtype=torch.float16))
    b = Q8Matrix(-a.codes, 2 * a.scales)
    il = Q8Matrix.interleave(a, b)
    assert torch.equal(il.codes[0:8], a.codes[0:8]) and torch.equal(il.codes[8:16], b.codes[0:8])
    assert torch.equal(il.codes[16:24], a.codes[8:16])
    assert torch.equal(il.scales[8:16], b.scales[0:8])
