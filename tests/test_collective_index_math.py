"""The collective kernels' work split, restated on the host (csrc/comm.cu: chunk_bounds,
cta_slice, the two-shot phases and the NVLS all-reduce / reduce-scatter loops): for
every world size up to 8, CTA count and awkward length or start offset, each element is
reduced by exactly one (rank, CTA) and every rank gathers every element once.  The
8-rank NVLS paths run here even where no 8-GPU measurement exists."""
import itertools

import pytest


def chunk_bounds(n, W, c):
    base, extra = divmod(n, W)
    lo = c * base + min(c, extra)
    return lo, lo + base + (1 if c < extra else 0)


def cta_slice(lo, hi, grid, b):
    per = (((hi - lo) + grid - 1) // grid + 63) & ~63
    a = min(hi, lo + b * per)
    return a, min(hi, a + per)


def comm_blocks(nbytes, want=0):
    return min(want, 160) if want > 0 else max(1, min(64, (nbytes + 65535) // 65536))


def lean_blocks(nbytes, want=0, sms=148):
    return min(want, 160) if want > 0 else max(1, min(sms, 160, (nbytes + 16383) // 16384))


LENGTHS = [0, 1, 3, 4, 5, 7, 63, 64, 65, 1000, 4099, 12345, 65536 + 3, (1 << 20) + 7]


def _grids(nbytes):
    return sorted({comm_blocks(nbytes), lean_blocks(nbytes), 128, 1})


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_two_shot_reduce_and_gather_cover_every_element_once(W):
    for n, esz in itertools.product(LENGTHS, (4, 2)):
        for grid in _grids(n * esz):
            count = [0] * n
            for r in range(W):
                lo, hi = chunk_bounds(n, W, r)
                for b in range(grid):
                    a, e = cta_slice(lo, hi, grid, b)
                    for i in range(a, e):
                        count[i] += 1
            assert all(c == 1 for c in count), (W, n, grid)
            # gather phase of one rank: chunk p of every rank p
            seen = [0] * n
            for p in range(W):
                lo, hi = chunk_bounds(n, W, p)
                for b in range(grid):
                    a, e = cta_slice(lo, hi, grid, b)
                    for i in range(a, e):
                        seen[i] += 1
            assert all(c == 1 for c in seen)


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_nvls_allreduce_split_covers_every_element_once(W):
    for n in LENGTHS:
        for esz, offsets in ((4, (0, 4, 8, 12)), (2, (0,))):
            if esz == 2 and n % 8:
                continue  # the host sends bf16 that is not whole 16-byte vectors to two-shot
            per_vec = 16 // esz
            for off in offsets:
                head = min(n, ((16 - (off & 15)) & 15) // esz)
                nvec = (n - head) // per_vec
                tail = head + nvec * per_vec
                for grid in _grids(n * esz):
                    count = [0] * n
                    for r in range(W):
                        lo, hi = chunk_bounds(nvec, W, r)
                        for b in range(grid):
                            a, e = cta_slice(lo, hi, grid, b)
                            for v in range(a, e):
                                for i in range(head + v * per_vec, head + (v + 1) * per_vec):
                                    count[i] += 1
                            if esz == 4 and r == 0 and b == 0:  # scalar head and tail elements
                                for i in list(range(head)) + list(range(tail, n)):
                                    count[i] += 1
                    assert all(c == 1 for c in count), (W, n, esz, off, grid)
                    # every vector starts on a 16-byte boundary
                    assert (off + head * esz) % 16 == 0 or nvec == 0


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_nvls_reduce_scatter_covers_each_partition_once(W):
    for n in LENGTHS:
        for grid in (64, 1, 7):
            for r in range(W):
                lo, hi = chunk_bounds(n, W, r)
                vlo, vhi = (lo + 3) // 4, hi // 4
                count = {}
                if vlo < vhi:
                    for b in range(grid):
                        a, e = cta_slice(vlo, vhi, grid, b)
                        for v in range(a, e):
                            for i in range(4 * v, 4 * v + 4):
                                count[i] = count.get(i, 0) + 1
                h_end = vlo * 4 if vlo < vhi else hi
                t_beg = vhi * 4 if vlo < vhi else hi
                for i in list(range(lo, h_end)) + list(range(t_beg, hi)):
                    count[i] = count.get(i, 0) + 1
                assert sorted(count) == list(range(lo, hi)), (W, n, r)
                assert all(c == 1 for c in count.values())
