"""Host-side checks of the peer-sharded gradient exchange's layout (no GPU):
the chunks tile each rank's gradient area exactly, in exchange (backward)
order, every shard is 256-byte aligned, each tensor-core layer's dW is cut
into the requested row blocks where its shape allows, and the region holds the six
areas plus the flag words.  The copies of the exchange index only through
these offsets, so an overlap or gap here would be a wrong copy on the GPU."""
import pytest

from ferrograd_b200 import FerroError, peer_layout


def _pad(n, u):
    return (n + u - 1) // u * u


@pytest.mark.parametrize("dims", [(4096, 4096, 4096, 10), (512, 256, 256, 10), (784, 128, 10),
                                  (64, 32, 10), (48, 40, 24, 10), (4096, 10)])
@pytest.mark.parametrize("nranks", [2, 3, 4, 8])
@pytest.mark.parametrize("chunks", [1, 2, 4, 8])
def test_chunks_tile_the_gradient_area(dims, nranks, chunks):
    region, ch = peer_layout(dims, nranks, chunks)
    unit = 64 * nranks
    nl = len(dims) - 1
    # expected per-layer buckets (forward order), then reversed for the exchange
    off, buckets = 0, []
    for l in range(nl):
        o, i = dims[l + 1], dims[l]
        raw = _pad(o * i, 64) + _pad(o, 64) + (64 if l == 0 else 0)
        buckets.append((off, _pad(raw, unit)))
        off += _pad(raw, unit)
    grad = off
    for off_c, len_c in ch:
        assert len_c > 0 and len_c % unit == 0 and off_c % unit == 0
        assert off_c + len_c <= grad
    # chunks of each layer are contiguous and cover its bucket; layers in
    # backward order; a layer's dW row blocks are equal where it is split
    pos = 0
    for l in reversed(range(nl)):
        b0, blen = buckets[l]
        o, i = dims[l + 1], dims[l]
        splittable = (chunks > 1 and o > 16 and o % chunks == 0 and (o // chunks) % 32 == 0
                      and ((o // chunks) * i) % unit == 0)
        first, cur = pos, b0
        while pos < len(ch) and cur < b0 + blen:
            assert ch[pos][0] == cur
            cur += ch[pos][1]
            pos += 1
        assert cur == b0 + blen, (l, cur, b0 + blen)
        assert pos - first == (chunks if splittable else 1), (l, pos - first)
        if splittable:
            for k in range(chunks - 1):
                assert ch[first + k][1] == (o // chunks) * i
    assert pos == len(ch)
    flags = _pad(2 * len(ch) * 8, 64)
    assert region == 6 * grad + flags


def test_bad_rank_counts_are_rejected():
    for n in (0, 1, 9):
        with pytest.raises(FerroError):
            peer_layout((512, 256, 10), n, 4)
    with pytest.raises(FerroError):
        peer_layout((512, 256, 10), 2, 9)
