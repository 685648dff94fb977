"""Collectives captured in a CUDA graph (csrc/comm.cu, device-resident flag epochs).

A one-rank NVLink group runs the real two-shot kernel (the world-size-1 shortcut in
``NVLinkGroup.allreduce`` is bypassed by calling the engine directly), so these run
on a single GPU: no kernel ever waits for another launch.  Checked against plain
fp32/fp64 PyTorch: the in-place result, the published sums of squares and their
fixed-order total, and that every launch - eager or replayed - advances the device
epoch counter by the epochs it used, so replays never reuse an epoch.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

TWO_SHOT_EPOCHS = 3


def _group():
    from dtrain_b200.parallel.nvlink import NVLinkGroup
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    return NVLinkGroup(0, 1, dev, lambda key, payload: [payload], timeout=5.0)


@pytest.mark.parametrize("lean", [False, True])
def test_twoshot_replays_in_a_graph_with_fresh_epochs(lean):
    pg = _group()
    try:
        n = (1 << 20) + 37
        buf = pg.alloc(n, torch.float32)
        x = torch.randn(n, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
        blocks = pg.collective_blocks(n * 4, lean=lean)
        stride = blocks + 3
        pad = pg.alloc(stride, torch.float64)
        tot = torch.zeros(1, dtype=torch.float64, device="cuda")
        scale = 0.5

        def launch():
            pg._eng.allreduce_inplace(buf, 0, scale, blocks, lean, pad, 2, stride)
            pg.sq_total(pad, tot, stride, 2, 2 + blocks)

        buf.copy_(x)
        e0 = pg.epoch
        launch()                                   # eager
        torch.cuda.synchronize()
        pg.check()
        assert pg.epoch == e0 + TWO_SHOT_EPOCHS
        ref = (x * scale).double()
        torch.testing.assert_close(buf, x * scale, rtol=0, atol=0)
        torch.testing.assert_close(tot[0], (ref * ref).sum(), rtol=1e-12, atol=0)

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                launch()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        e1 = pg.epoch
        assert e1 == e0 + TWO_SHOT_EPOCHS  # capturing launches nothing
        for k in range(1, 4):
            buf.copy_(x)
            g.replay()
            torch.cuda.synchronize()
            pg.check()
            assert pg.epoch == e1 + k * TWO_SHOT_EPOCHS
            torch.testing.assert_close(buf, x * scale, rtol=0, atol=0)
            torch.testing.assert_close(tot[0], (ref * ref).sum(), rtol=1e-12, atol=0)
        # eager calls and replays share the counter
        buf.copy_(x)
        launch()
        g.replay()
        torch.cuda.synchronize()
        pg.check()
        assert pg.epoch == e1 + 5 * TWO_SHOT_EPOCHS
        torch.testing.assert_close(buf, x * scale * scale, rtol=0, atol=0)
        del g
    finally:
        pg.close()


def test_sq_total_is_a_fixed_order_sum_over_ranks_and_slots():
    pg = _group()
    try:
        from dtrain_b200.ops._ext import lib
        stride, world = 300, 3
        pad = torch.randn(world * stride, dtype=torch.float64, device="cuda")
        out = torch.zeros(1, dtype=torch.float64, device="cuda")
        lib().sq_total(pad, out, world, stride, 10, 250)
        want = pad.reshape(world, stride)[:, 10:250].sum()
        torch.testing.assert_close(out[0], want, rtol=1e-13, atol=1e-13)
        again = torch.zeros_like(out)
        lib().sq_total(pad, again, world, stride, 10, 250)
        assert torch.equal(out, again)
        with pytest.raises(RuntimeError, match="do not fit"):
            lib().sq_total(pad, out, world, stride, 10, stride + 1)
    finally:
        pg.close()
