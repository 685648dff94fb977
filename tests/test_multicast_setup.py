"""Host-side set-up of an NVSwitch multicast mapping (``SymmetricBuffer._map_multicast``),
with the driver calls replaced by a fake: every rank joins the object, the ranks vote
over the bootstrap exchange, and only a unanimous join goes on to bind - a rank whose
join failed must not leave the others blocked in a bind that waits for the whole team."""
import os

import pytest

from dtrain_b200.parallel import nvlink
from dtrain_b200.utils.store import CommError


class FakeDriver:
    def __init__(self, join_error=None):
        self.calls = []
        self.join_error = join_error

    def mc_create(self, size, world):
        self.calls.append(("create", size, world))
        return 77, os.open(os.devnull, os.O_RDONLY)

    def mc_import(self, fd):
        self.calls.append(("import",))
        return 77

    def mc_add_device(self, mc):
        self.calls.append(("join", mc))
        if self.join_error:
            raise RuntimeError(self.join_error + "\nmore lines")

    def mc_release(self, mc):
        self.calls.append(("release", mc))

    def mc_bind_map(self, mc, ptr, size, world):
        self.calls.append(("bind", mc, ptr, size, world))
        return 0xABC000


class FakeFdx:
    def broadcast(self, fd, size, root=0):
        if fd is None:
            return os.open(os.devnull, os.O_RDONLY), 1 << 21
        return None


class FakeGroup:
    def __init__(self, rank, votes):
        self.rank, self.world = rank, 2
        self._fdx = FakeFdx()
        self._mc_joins = 0
        self.keys = []
        self._votes = votes

    def _exchange(self, key, payload):
        self.keys.append((key, payload))
        v = list(self._votes)
        v[self.rank] = payload
        return v


def _map(monkeypatch, driver, group):
    monkeypatch.setattr(nvlink, "lib", lambda: driver)
    buf = object.__new__(nvlink.SymmetricBuffer)
    buf.ptr = 0x1000
    return buf._map_multicast(group, 1 << 21)


@pytest.mark.parametrize("rank", [0, 1])
def test_unanimous_join_binds_and_maps(monkeypatch, rank):
    drv = FakeDriver()
    g = FakeGroup(rank, [b"", b""])
    assert _map(monkeypatch, drv, g) == 0xABC000
    assert ("join", 77) in drv.calls
    assert drv.calls[-1] == ("bind", 77, 0x1000, 1 << 21, 2)
    assert g.keys == [("mc-join/1", b"")]


def test_a_peer_that_could_not_join_stops_every_rank_before_the_bind(monkeypatch):
    drv = FakeDriver()
    g = FakeGroup(0, [b"", b"vmm: cuMulticastAddDevice failed with code 801"])
    with pytest.raises(CommError, match="could not join"):
        _map(monkeypatch, drv, g)
    assert ("release", 77) in drv.calls
    assert not any(c[0] == "bind" for c in drv.calls)


def test_own_failed_join_is_reported_and_nothing_is_bound(monkeypatch):
    drv = FakeDriver(join_error="vmm: cuMulticastAddDevice failed with code 801")
    g = FakeGroup(1, [b"", b""])
    with pytest.raises(CommError, match="code 801"):
        _map(monkeypatch, drv, g)
    assert g.keys == [("mc-join/1", b"vmm: cuMulticastAddDevice failed with code 801")]
    assert ("release", 77) in drv.calls and not any(c[0] == "bind" for c in drv.calls)
