"""Per-GPU NVLink accounting of one sync, shared by the benchmark's roofline and the dry-run
planner.  A route is ``{"src": gpu, "dst": [gpu, ...], "bytes": n, "multicast": bool}``: the
bytes one program stores for one receiver (unicast) or for a replica group at once (multicast).
"""
from __future__ import annotations


def link_bytes(routes: list[dict]) -> tuple[dict, dict, dict, int]:
    """Per-GPU unicast egress, multicast egress and ingress bytes, and the bytes that stay on one
    GPU.  A unicast route to its own GPU stays in HBM; a multicast store leaves its sender's GPU
    once and the NVSwitch delivers it to every replica's GPU (its own included)."""
    egress: dict[int, int] = {}
    mc_egress: dict[int, int] = {}
    ingress: dict[int, int] = {}
    local = 0
    for r in routes:
        n, src = int(r["bytes"]), int(r["src"])
        remote = list(r["dst"]) if r["multicast"] else [d for d in r["dst"] if d != src]
        local += n * (len(r["dst"]) - len(remote))
        if not remote:
            continue
        if r["multicast"]:
            mc_egress[src] = mc_egress.get(src, 0) + n
        else:
            egress[src] = egress.get(src, 0) + n * len(remote)
        for d in remote:
            ingress[d] = ingress.get(d, 0) + n
    return egress, mc_egress, ingress, local


def busiest_link(routes: list[dict], peer_gbs: float, mc_gbs: float) -> tuple[str, int, float] | None:
    """(``"egress"`` or ``"ingress"``, GPU, ideal ms) of the GPU whose NVLink traffic takes
    longest: unicast egress and ingress at ``peer_gbs``, multicast egress at ``mc_gbs``.  None
    when every byte stays on its GPU."""
    egress, mc_egress, ingress, _local = link_bytes(routes)
    times = [(("egress", d), egress.get(d, 0) / peer_gbs + mc_egress.get(d, 0) / mc_gbs)
             for d in set(egress) | set(mc_egress)]
    times += [(("ingress", d), b / peer_gbs) for d, b in ingress.items()]
    if not times:
        return None
    (side, dev), t = max(times, key=lambda x: (x[1], x[0][0] == "egress"))
    return side, dev, t / 1e6
