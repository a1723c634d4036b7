"""Per-GPU NVLink accounting of a sync (``utils/links.py``): the model behind the benchmark's
roofline and the dry-run planner's estimate."""
from weightbridge_b200.utils.links import busiest_link, link_bytes


def _r(src, dst, n, mc=False):
    return {"src": src, "dst": list(dst), "bytes": n, "multicast": mc}


def test_local_routes_stay_in_hbm():
    eg, mc, ing, local = link_bytes([_r(0, [0], 100), _r(1, [1], 50)])
    assert eg == {} and mc == {} and ing == {} and local == 150
    assert busiest_link([_r(0, [0], 100)], 800.0, 500.0) is None


def test_unicast_fanout_counts_each_remote_copy():
    eg, mc, ing, local = link_bytes([_r(0, [1, 2], 10), _r(0, [0], 5)])
    assert eg == {0: 20} and ing == {1: 10, 2: 10} and local == 5


def test_multicast_leaves_once_and_reaches_its_own_gpu_through_the_switch():
    eg, mc, ing, local = link_bytes([_r(0, [0, 1, 2], 10, mc=True)])
    assert eg == {} and mc == {0: 10} and ing == {0: 10, 1: 10, 2: 10} and local == 0


def test_busiest_link_weighs_multicast_at_its_own_rate():
    # 8e8 bytes multicast at 400 GB/s (2 ms) beats 8e8 bytes of ingress at 800 GB/s (1 ms)
    side, gpu, ms = busiest_link([_r(0, [1, 2], int(8e8), mc=True)], 800.0, 400.0)
    assert (side, gpu) == ("egress", 0) and abs(ms - 2.0) < 1e-9
    # unicast egress and multicast egress of one GPU add up
    side, gpu, ms = busiest_link([_r(0, [1, 2], int(4e8), mc=True), _r(0, [3], int(8e8))], 800.0, 400.0)
    assert (side, gpu) == ("egress", 0) and abs(ms - 2.0) < 1e-9
    # many senders into one GPU: ingress bound
    side, gpu, ms = busiest_link([_r(s, [4], int(4e8)) for s in range(4)], 800.0, 400.0)
    assert (side, gpu) == ("ingress", 4) and abs(ms - 2.0) < 1e-9
