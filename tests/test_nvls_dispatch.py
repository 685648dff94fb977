"""Host-side dispatch of ``NVLinkGroup.allreduce(method="nvls")`` with the native engine
replaced by a recorder (no GPU): in-place launches on multicast-mapped tensors,
staging for other tensors, the two-shot fallback for bf16 that is not whole 16-byte
vectors, and the refusals (a group without multicast; lean or sum-of-squares calls on
staged tensors)."""
import pytest
import torch

from dtrain_b200.parallel import nvlink


class Engine:
    def __init__(self, mapped):
        self.mapped, self.calls = mapped, []

    def has_multicast(self, t):
        return any(t.data_ptr() >= m.data_ptr() and t.data_ptr() < m.data_ptr() + m.numel() * m.element_size()
                   for m in self.mapped)

    def allreduce_nvls(self, t, scale, blocks, lean, pad, base, stride):
        self.calls.append(("nvls", t.data_ptr(), t.numel(), scale, blocks, lean, base, stride))
        t.mul_(2.0 * scale)  # stands for the sum over two ranks holding the same values


class Stage:
    def __init__(self, nbytes):
        self.buf = torch.zeros(nbytes, dtype=torch.uint8)
        self.nbytes = nbytes

    def tensor(self, n, dtype, byte_offset=0):
        return self.buf[byte_offset:].view(dtype)[:n]


def _group(mapped, nvls=True):
    g = object.__new__(nvlink.NVLinkGroup)
    g.world, g.rank, g.nvls, g.blocks, g.seq = 2, 0, nvls, 0, 0
    g._eng = Engine(mapped)
    g._staging = None
    g.staged = []

    def stage(nbytes):
        g._staging = Stage(nbytes)
        g.staged.append(nbytes)
        return g._staging

    g._stage = stage
    g.twoshot = []

    def allreduce(t, algo="ring", scale=1.0, method="auto", blocks=0, lean=False, sq=None):
        if method == "twoshot":
            g.twoshot.append(t.numel())
            return t
        return nvlink.NVLinkGroup.allreduce(g, t, algo, scale, method, blocks, lean, sq)

    g.allreduce = allreduce
    return g


def test_mapped_tensor_runs_in_place_with_its_options():
    buf = torch.ones(1000)
    g = _group([buf])
    pad = torch.zeros(8, dtype=torch.float64)
    g.allreduce(buf[4:], method="nvls", scale=0.5, blocks=3, lean=True, sq=(pad, 2, 4))
    assert g._eng.calls == [("nvls", buf[4:].data_ptr(), 996, 0.5, 3, True, 2, 4)]
    assert g.seq == 1 and not g.staged
    assert torch.equal(buf[4:], torch.ones(996)) and buf[0] == 1.0


def test_other_tensors_go_through_the_multicast_staging_buffer():
    g = _group([])
    x = torch.arange(10, dtype=torch.float32)
    g.allreduce(x, method="nvls", scale=1.0)
    assert g.staged == [40]
    assert torch.equal(x, 2.0 * torch.arange(10, dtype=torch.float32))  # copied back


def test_bf16_that_is_not_whole_vectors_falls_back_to_two_shot():
    buf = torch.ones(1003, dtype=torch.bfloat16)
    g = _group([buf])
    g.allreduce(buf, method="nvls")
    assert g.twoshot == [1003] and not g._eng.calls


def test_refusals():
    with pytest.raises(ValueError, match="nvls=True"):
        _group([], nvls=False).allreduce(torch.ones(8), method="nvls")
    g = _group([])
    with pytest.raises(ValueError, match="needs a tensor from alloc"):
        g.allreduce(torch.ones(8), method="nvls", lean=True)
