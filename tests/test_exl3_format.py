"""EXL3 checkpoint format: decoder vs a bit-by-bit scalar decode, state-dict round trip, H128."""

import random

import torch

from vllm_cmp170hx_b200.formats import exl3 as fx


def _scalar(tr, bits_x2, cb, k, n):
    r, c = k & 15, n & 15
    lane = (c & 7) * 4 + ((r & 7) >> 1)
    idx = lane * 8 + (r & 1) + 2 * (r >> 3) + 4 * (c >> 3)
    end = (idx + 1) * (bits_x2 // 2) + (((idx + 1) // 2) if bits_x2 & 1 else 0)
    ring = 128 * bits_x2
    start = (end - 16 + ring) % ring
    e = [int(v) & 0xFFFF for v in tr[k // 16, n // 16].tolist()]
    bits = []
    for w in range(ring // 32):
        word = e[2 * w] | (e[2 * w + 1] << 16)
        bits += [(word >> (31 - i)) & 1 for i in range(32)]
    st = 0
    for i in range(16):
        st = (st << 1) | bits[(start + i) % ring]
    return float(fx.codebook_value(torch.tensor([st]), cb)[0])


def test_decoder_matches_scalar_definition():
    g = torch.Generator().manual_seed(0)
    rnd = random.Random(0)
    for bits_x2, cb in [(8, 2), (8, 1), (4, 2), (6, 1), (5, 2), (3, 2), (7, 2), (16, 1), (2, 1)]:
        m = fx.random_matrix(128, 128, bits_x2, cb, generator=g)
        W = fx.decode_weight(m.trellis, bits_x2, cb)
        for _ in range(24):
            k, n = rnd.randrange(128), rnd.randrange(128)
            assert float(W[k, n]) == _scalar(m.trellis, bits_x2, cb, k, n)


def test_codebook_known_values():
    # state 0: codebook 2 -> fma16(1024 + 0, 0x1eee, 0xc931); codebook 1 -> 0x3b60 + 0x3b60 as fp16
    v2 = float(fx.codebook_value(torch.tensor([0]), 2)[0])
    a = torch.tensor([0x6400], dtype=torch.int16).view(torch.float16).double()
    b = torch.tensor([0x1EEE], dtype=torch.int16).view(torch.float16).double()
    c = torch.tensor([0xC931 - 65536], dtype=torch.int16).view(torch.float16).double()
    assert v2 == float((a * b + c).to(torch.float16))
    v1 = float(fx.codebook_value(torch.tensor([0]), 1)[0])
    h = torch.tensor([0x3B60], dtype=torch.int16).view(torch.float16)
    assert v1 == float(h + h)


def test_state_dict_round_trip():
    g = torch.Generator().manual_seed(1)
    m = fx.random_matrix(256, 128, 8, 2, generator=g)
    sd = m.state_dict("model.layers.0.mlp.experts.3.down_proj")
    m2 = fx.Exl3Matrix.from_state_dict(sd, "model.layers.0.mlp.experts.3.down_proj")
    assert torch.equal(m.trellis, m2.trellis) and m2.bits_x2 == 8 and m2.codebook == 2


def test_hadamard_orthonormal():
    x = torch.randn(3, 256, dtype=torch.float64)
    y = fx.hadamard128(fx.hadamard128(x)).double()
    assert torch.allclose(y, x.float().double(), atol=1e-5)
    H = fx.hadamard128(torch.eye(128))
    assert torch.allclose(H @ H.t(), torch.eye(128), atol=1e-5)
