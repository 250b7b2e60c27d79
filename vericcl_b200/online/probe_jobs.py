"""Calibration probe planning and probe schedules.

A probe job is a tiny schedule that exercises one primitive component, or a
concurrency mode of several, on the real GPUs:

* ``send:s:d:c`` — a transfer s→d over ``c`` channels (link component);
* ``rrc:s:d:c``  — a receive-reduce-copy s→d (rrc component);
* ``copy:r`` / ``reduce:r`` — local copy / reduce on rank r;
* shared modes — two or more flows that share a resource (NVLink port, NIC),
  measured together so the model gets a measured rate vector.

Each job carries at least three payload sizes around the request's slice
size (or the configured ``payload_sizes``).  ``build_probe_xml`` emits the
job as MSCCL-style XML, so probes run through exactly the same compiler and
interpreter as real schedules (reference: vericcl/verification/online/
probe_jobs.py:16-216, probe_xml.py:13).
"""
from __future__ import annotations

from dataclasses import dataclass
from itertools import combinations

PRIORITY = {"link_intra": 0, "local": 1, "link_inter": 2, "shared": 3}


@dataclass(frozen=True)
class ProbeFlow:
    kind: str          # send | rrc | copy | reduce
    src: int
    dst: int
    channels: int = 1

    @property
    def flow_id(self) -> str:
        if self.kind in ("copy", "reduce"):
            return "%s:%d" % (self.kind, self.src)
        return "%s:%d:%d:c%d" % (self.kind, self.src, self.dst, self.channels)

    @property
    def component(self) -> str:
        if self.kind in ("copy", "reduce"):
            return "%s:%d" % (self.kind, self.src)
        return ("link:" if self.kind == "send" else "rrc:") + "%d:%d" % (self.src, self.dst)


@dataclass(frozen=True)
class ProbeJob:
    job_id: str
    group: str
    flows: tuple
    payload_sizes: tuple
    mode: str = "single"          # single | shared
    resources: tuple = ()

    def as_json(self):
        return {"job_id": self.job_id, "group": self.group, "mode": self.mode, "resources": list(self.resources),
                "payload_sizes": list(self.payload_sizes),
                "flows": [{"kind": f.kind, "src": f.src, "dst": f.dst, "channels": f.channels} for f in self.flows]}


def payload_sizes(request, explicit=()):
    """At least three legal sizes around S (whole elements, multiples of 16 bytes)."""
    if explicit:
        return tuple(sorted(set(explicit)))
    s = request.hyperparameters.slice_size_bytes or request.hyperparameters.total_size_bytes
    unit = max(16, request.element_bytes)
    sizes = {max(unit, (int(s * f) // unit) * unit) for f in (0.25, 0.5, 1.0, 2.0)}
    return tuple(sorted(sizes))


def link_classes(topology) -> dict:
    """Interchangeable links: same α, β, same/other node, and the same kinds of shared resources on them.

    Returns ``{class key: [LinkKey, ...]}`` with members in (src, dst) order.
    """
    classes = {}
    for key, link in sorted(topology.links.items()):
        kinds = tuple(sorted(topology.resources[r].kind if r in topology.resources else r.split("-")[0]
                             for r in link.resource_ids))
        same_node = topology.node_of(key.src).node_id == topology.node_of(key.dst).node_id
        classes.setdefault((same_node, link.alpha_us, link.beta_us_per_byte, kinds), []).append(key)
    return classes


def representatives(topology, per_class: int = 2) -> tuple:
    """(links to probe, {probed component suffix "s:d": [suffixes it stands for]}, ranks to probe).

    Representatives of a class are spread over different source ranks; each
    stands for the members nearest to it in the class order.  One rank per
    node represents the node's local copy/reduce.
    """
    chosen, stands_for = [], {}
    for members in link_classes(topology).values():
        picks, seen_src = [], set()
        for key in members:
            if key.src not in seen_src:
                picks.append(key)
                seen_src.add(key.src)
            if len(picks) == per_class:
                break
        for i, key in enumerate(members):
            rep = picks[i * len(picks) // len(members)]
            stands_for.setdefault("%d:%d" % (rep.src, rep.dst), []).append("%d:%d" % (key.src, key.dst))
        chosen.extend(picks)
    ranks = sorted({node.ranks[0] for node in topology.nodes if node.ranks})
    return tuple(chosen), stands_for, tuple(ranks)


def plan_probes(request, topology, *, max_channels: int = 1, include_shared: bool = True):
    cfg = request.request_config["sketch"]["calibration"]
    sizes = payload_sizes(request, cfg["payload_sizes"])
    jobs = []
    reducing = request.collective.reducing
    if cfg.get("probe_scope", "every_link") == "link_classes":
        links, _, local_ranks = representatives(topology)
        link_items = [(k, topology.links[k]) for k in sorted(links)]
    else:
        link_items, local_ranks = sorted(topology.links.items()), tuple(range(topology.rank_count))
    for key, link in link_items:
        same_node = topology.node_of(key.src).node_id == topology.node_of(key.dst).node_id
        group = "link_intra" if same_node else "link_inter"
        for c in range(1, max_channels + 1):
            jobs.append(ProbeJob("send-%d-%d-c%d" % (key.src, key.dst, c), group,
                                 (ProbeFlow("send", key.src, key.dst, c),), sizes))
            if reducing:
                jobs.append(ProbeJob("rrc-%d-%d-c%d" % (key.src, key.dst, c), group,
                                     (ProbeFlow("rrc", key.src, key.dst, c),), sizes))
    for r in local_ranks:
        jobs.append(ProbeJob("copy-%d" % r, "local", (ProbeFlow("copy", r, r),), sizes))
        if reducing:
            jobs.append(ProbeJob("reduce-%d" % r, "local", (ProbeFlow("reduce", r, r),), sizes))
    if include_shared:
        kinds_done = set()
        for rid, res in sorted(topology.resources.items()):
            members = sorted(res.links)
            if len(members) < 2:
                continue
            if cfg.get("probe_scope", "every_link") == "link_classes":
                # one resource of each class (kind, capacity, number of member links) stands for the others:
                # a group's NIC and a rank's share of it are both NICs, but not interchangeable
                cls = (res.kind, round(float(res.capacity_bytes_per_us), 6), len(members))
                if cls in kinds_done:
                    continue
                kinds_done.add(cls)
            pairs = list(combinations(members, 2))[:2]
            for i, (a, b) in enumerate(pairs):
                jobs.append(ProbeJob("shared-%s-%d" % (rid, i), "shared",
                                     (ProbeFlow("send", a.src, a.dst), ProbeFlow("send", b.src, b.dst)), sizes,
                                     "shared", (rid,)))
    jobs.sort(key=lambda j: (PRIORITY[j.group], j.job_id))
    return jobs


def build_probe_xml(job: ProbeJob, ranks: int) -> str:
    """MSCCL-style XML running every flow of ``job`` concurrently on one chunk each."""
    nflows = len(job.flows)
    tbs = {r: [] for r in range(ranks)}
    for i, f in enumerate(job.flows):
        if f.kind in ("send", "rrc"):
            tbs[f.src].append(("send", f.dst, i, '<step s="0" type="s" srcbuf="i" srcoff="%d" dstbuf="o" '
                               'dstoff="%d" cnt="1" depid="-1" deps="-1" hasdep="0"/>' % (i, i)))
            kind = "rrc" if f.kind == "rrc" else "r"
            src = 'srcbuf="i" srcoff="%d"' % i if kind == "rrc" else 'srcbuf="o" srcoff="%d"' % i
            tbs[f.dst].append(("recv", f.src, i, '<step s="0" type="%s" %s dstbuf="o" dstoff="%d" cnt="1" '
                               'depid="-1" deps="-1" hasdep="0"/>' % (kind, src, i)))
        elif f.kind == "copy":
            tbs[f.src].append(("local", -1, i, '<step s="0" type="cpy" srcbuf="i" srcoff="%d" dstbuf="o" '
                               'dstoff="%d" cnt="1" depid="-1" deps="-1" hasdep="0"/>' % (i, i)))
        else:
            tbs[f.src].append(("local", -1, i, '<step s="0" type="re" srcbuf="i" srcoff="%d" dstbuf="o" '
                               'dstoff="%d" cnt="1" depid="-1" deps="-1" hasdep="0"/>' % (i, i)))
    lines = ['<algo name="probe-%s" nchannels="1" nchunksperloop="%d" proto="Simple" coll="allreduce" '
             'inplace="0" redop="nop" ngpus="%d" minBytes="0" maxBytes="0">' % (job.job_id, nflows, ranks)]
    for r in range(ranks):
        lines.append('  <gpu id="%d" i_chunks="%d" o_chunks="%d" s_chunks="0">' % (r, nflows, nflows))
        for t, (direction, peer, i, step) in enumerate(tbs[r]):
            send = peer if direction == "send" else -1
            recv = peer if direction == "recv" else -1
            lines.append('    <tb id="%d" send="%d" recv="%d" chan="%d">' % (t, send, recv, i))
            lines.append("      " + step)
            lines.append("    </tb>")
        lines.append("  </gpu>")
    lines.append("</algo>")
    return "\n".join(lines) + "\n"
