"""Host header of the device activation ring (a supervisor's view without touching the GPUs)."""

from saelens_b200.parallel.device_ring import HostRingHeader


def test_host_ring_header_counts_per_rank(tmp_path):
    path = tmp_path / "hdr"
    a = HostRingHeader(path, world=3, rank=0, create=True)
    b = HostRingHeader(path, world=3, rank=2, create=False)
    a.add("written", 2)
    b.add("taken")
    b.add("taken")
    a.set("done", 1)
    snap = HostRingHeader(path, world=3, rank=1, create=False).snapshot()
    assert snap == {"written": [2, 0, 0], "taken": [0, 0, 2], "done": [1, 0, 0]}
