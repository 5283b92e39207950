"""The data-movement operators at sizes of whole layers (48k+ rows) against
the oracle.  lrk_compact, lrk_append and lrk_batch_append take the bulk-copy
kernel (bulk_kernel in csrc/move.cu: outputs of at least 2 x SMs x 64 rows,
16-byte aligned rows of 16-byte multiples up to 512 bytes, at most one run
break per tile on average) in the aligned cases and the vector gather engine
in the misaligned twins and heavy compactions; merge, merge_layers and the
legacy flattened append / compact run the vector engine at the same sizes.
Row widths 128, 256 and 512 bytes; runs of every length (compactions remove
runs and isolated rows; merges interleave single recalled rows)."""
import numpy as np
import pytest

from oracle import lrk_oracle as O

pytestmark = pytest.mark.gpu

ROWS = 48_000  # > 2 x 148 x 64


@pytest.fixture(scope="module")
def C(cuda):
    from code_for_iclr27_b200 import operators

    return operators()


def bits(t):
    import torch

    return t.cpu().view(torch.int16).numpy()


def kv(rows, d, g, device, misaligned=False):
    """bf16 [rows, d] on the device; misaligned: 2 bytes past a 16-byte boundary."""
    import torch

    data = torch.randn(rows * d + 1, generator=g).to(torch.bfloat16).to(device)
    return data[1:].view(rows, d) if misaligned else data[:rows * d].view(rows, d)


@pytest.mark.parametrize("d,misaligned", [(64, False), (128, False), (256, False), (128, True)])
def test_append_bulk(C, cuda, d, misaligned):
    import torch

    g = torch.Generator().manual_seed(d)
    lengths = [ROWS // 8 + 13 * h for h in range(8)]
    rows = sum(lengths)
    keys, values = kv(rows, d, g, cuda, misaligned), kv(rows, d, g, cuda, misaligned)
    positions = torch.arange(rows, dtype=torch.float32, device=cuda).reshape(-1, 1)
    nk = torch.randn(1, 8, 1, d, generator=g).to(torch.bfloat16).to(cuda)
    nv = torch.randn(1, 8, 1, d, generator=g).to(torch.bfloat16).to(cuda)
    cumulative = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int32, device=cuda)
    out = C.append(keys, values, positions, nk, nv, cumulative, 70000, max(lengths))
    expect = O.append(bits(keys), bits(values), positions.cpu().numpy(), bits(nk), bits(nv),
                      cumulative.cpu().numpy(), 70000)
    np.testing.assert_array_equal(bits(out[0]), expect[0])
    np.testing.assert_array_equal(bits(out[1]), expect[1])
    np.testing.assert_array_equal(out[2].cpu().numpy(), expect[2])


@pytest.mark.parametrize("d,misaligned", [(64, False), (128, False), (256, False), (128, True)])
def test_compact_bulk(C, cuda, d, misaligned):
    import torch

    g = torch.Generator().manual_seed(10 + d)
    rows = ROWS + 777
    keys, values = kv(rows, d, g, cuda, misaligned), kv(rows, d, g, cuda, misaligned)
    positions = (torch.arange(rows, dtype=torch.float32) * 2).reshape(-1, 1).to(cuda)
    # At most one removed row per 64-row tile on average takes the bulk kernel
    # (runs of every length, several per tile in places); more, the vector engine.
    for removed in (torch.randperm(rows, generator=g)[:500].sort().values,
                    torch.randperm(rows, generator=g)[:rows // 7].sort().values,
                    torch.cat([torch.arange(5, 70), torch.arange(1000, 1001), torch.arange(rows - 130, rows)]),
                    torch.zeros(0, dtype=torch.int64)):
        out = C.compact(keys, values, positions, removed.to(cuda))
        expect = O.compact(bits(keys), bits(values), positions.cpu().numpy(), removed.numpy())
        np.testing.assert_array_equal(bits(out[0]), expect[0])
        np.testing.assert_array_equal(bits(out[1]), expect[1])
        np.testing.assert_array_equal(out[2].cpu().numpy(), expect[2])


@pytest.mark.parametrize("misaligned", [False, True])
def test_merge_and_merge_layers_bulk(C, cuda, misaligned):
    import torch

    g = torch.Generator().manual_seed(21)
    d, rows, recalled_rows = 128, ROWS, 3000
    keys, values = kv(rows, d, g, cuda, misaligned), kv(rows, d, g, cuda, misaligned)
    positions = torch.arange(rows, dtype=torch.float32).reshape(-1, 1).to(cuda)
    recalled = torch.randn(recalled_rows, 2, d, generator=g).to(torch.bfloat16).to(cuda)
    recalled_pos = (torch.arange(recalled_rows, dtype=torch.float32) + 0.5).to(cuda)
    # Resident rows in order with recalled rows spliced in at random places.
    slots = np.sort(np.random.default_rng(1).choice(rows + recalled_rows, recalled_rows, replace=False))
    mapping = np.empty(rows + recalled_rows, dtype=np.int64)
    resident = np.ones(rows + recalled_rows, dtype=bool)
    resident[slots] = False
    mapping[resident] = np.arange(rows)
    mapping[slots] = -np.arange(1, recalled_rows + 1)
    mapping_t = torch.as_tensor(mapping).to(cuda)
    out = C.merge(keys, values, positions, recalled, recalled_pos, mapping_t)
    expect = O.merge(bits(keys), bits(values), positions.cpu().numpy(), bits(recalled), recalled_pos.cpu().numpy(),
                     mapping)
    for got, exp in zip(out[:2], expect[:2]):
        np.testing.assert_array_equal(bits(got), exp)
    np.testing.assert_array_equal(out[2].cpu().numpy(), expect[2])
    layers = C.merge_layers([keys, keys], [values, values], [positions, positions], [recalled, recalled],
                            [recalled_pos, recalled_pos], [mapping_t, mapping_t])
    for i in range(2):
        for got, exp in zip((layers[0][i], layers[1][i]), expect[:2]):
            np.testing.assert_array_equal(bits(got), exp)
        np.testing.assert_array_equal(layers[2][i].cpu().numpy(), expect[2])


def test_batch_append_bulk(C, cuda):
    import torch

    g = torch.Generator().manual_seed(31)
    requests, heads, d = 3, 8, 128
    ks, vs, ps, lens = [], [], [], []
    for r in range(requests):
        hl = [ROWS // heads + 17 * h + r for h in range(heads)]
        n = sum(hl)
        ks.append(kv(n, d, g, cuda))
        vs.append(kv(n, d, g, cuda))
        ps.append((torch.arange(n, dtype=torch.float32) * 3).reshape(-1, 1).to(cuda))
        lens.append(hl)
    nk = torch.randn(requests, heads, 1, d, generator=g).to(torch.bfloat16).to(cuda)
    nv = torch.randn(requests, heads, 1, d, generator=g).to(torch.bfloat16).to(cuda)
    logical = [100000 + r for r in range(requests)]
    out = C.batch_append(ks, vs, ps, nk, nv, lens, logical)
    expect = O.batch_append([bits(k) for k in ks], [bits(v) for v in vs], [p.cpu().numpy() for p in ps],
                            bits(nk)[:, :, 0], bits(nv)[:, :, 0], lens, logical)
    for got, exp in zip(out, expect):
        np.testing.assert_array_equal(bits(got) if got.dtype == torch.bfloat16 else got.cpu().numpy(), exp)


def test_legacy_flattened_bulk(cuda):
    import torch

    from code_for_iclr27_b200 import legacy_operators

    L = legacy_operators()
    g = torch.Generator().manual_seed(41)
    d = 128
    head_lens = torch.tensor([ROWS // 4 + 5 * h for h in range(4)], dtype=torch.int32)
    cu = torch.cat([torch.zeros(1, dtype=torch.int32), head_lens.cumsum(0).to(torch.int32)])
    cache = kv(int(head_lens.sum()), d, g, cuda)
    states = torch.randn(2, 2, 2, d, generator=g).to(torch.bfloat16).to(cuda)
    out = L.append_flattened_cache(cache, states, head_lens.to(cuda), cu.to(cuda))
    np.testing.assert_array_equal(bits(out), O.append_flattened(bits(cache), bits(states), head_lens.numpy(),
                                                                cu.numpy()))
    keys, values = kv(ROWS, d, g, cuda), kv(ROWS, d, g, cuda)
    keep = torch.cat([torch.arange(0, ROWS // 2), torch.arange(ROWS - 5000, ROWS), torch.tensor([7, 7, 3])])
    ck, cv = L.compact_flattened_kv(keys, values, keep.to(cuda))
    ek, ev = O.compact_flattened(bits(keys), bits(values), keep.numpy())
    np.testing.assert_array_equal(bits(ck), ek)
    np.testing.assert_array_equal(bits(cv), ev)
