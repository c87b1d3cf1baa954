"""Host emulation of the fused collectives' schedules (CPU oracle for the device kernels).

Each function restates, in NumPy, the work partition and the phase order of
one device kernel: which CTA handles which vectors, which rank writes which
peer's inbox or outbox, where the barriers sit, and what is rounded to bf16 on
the wire. Running every rank and every CTA of a phase before the next phase
starts is exactly what the kernels' CTA-pairwise barriers guarantee, so the
emulated result must equal a plain reduction of the bf16-rounded inputs; the
tests check that for many shapes, and check the all-gather GEMM's chunk
schedule for coverage and order. The chunk-pipelined all-reduce is emulated
with ranks and CTAs interleaved at random, so its flag protocol (and buffer
reuse across launches) is checked for deadlocks and stale reads. (Device
counterparts: ``ar_twoshot_kernel``, ``ar_pipe_kernel``, ``ar_oneshot_kernel``,
``rs_push_kernel`` in csrc/comm.cu and ``AgGate::worker`` in csrc/ag_gemm.cu.)
"""

from __future__ import annotations

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 (nearest, ties to even) and return them as fp32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _cta_ranges(slice_vecs: int, ctas: int):
    """[v0, v1) of 8-element vectors per CTA, as the kernels split a slice (CTAs past the end get
    an empty range: they do no work but still take part in the barriers)."""
    per = (slice_vecs + ctas - 1) // ctas
    for b in range(ctas):
        v0 = b * per
        v1 = min(v0 + per, slice_vecs)
        if v1 > v0:
            yield b, v0, v1


def two_shot_allreduce(srcs: list[np.ndarray], ctas: int, scale: float) -> list[np.ndarray]:
    """Emulate ``ar_twoshot_kernel`` on every rank: fp32 in, bf16 on the wire, fp32 out."""
    world = len(srcs)
    n = srcs[0].size
    assert n % (8 * world) == 0
    slice_vecs = n // 8 // world
    sv = slice_vecs * 8                       # elements per slice
    inbox = [np.zeros(n, np.float32) for _ in range(world)]    # [src rank][slice] per owner
    outbox = [np.zeros(n, np.float32) for _ in range(world)]
    # phase 1: CTA b of rank r pushes its vectors of every slice s to owner s's inbox[r]
    for r in range(world):
        for _, v0, v1 in _cta_ranges(slice_vecs, ctas):
            for s in range(world):
                src = srcs[r][s * sv + v0 * 8: s * sv + v1 * 8]
                inbox[s][r * sv + v0 * 8: r * sv + v1 * 8] = bf16_round(src)
    # (barrier) phase 2: owner r reduces its slice and pushes the bf16 result to every outbox[q][r]
    for r in range(world):
        for _, v0, v1 in _cta_ranges(slice_vecs, ctas):
            acc = np.zeros((v1 - v0) * 8, np.float32)
            for q in range(world):
                acc += inbox[r][q * sv + v0 * 8: q * sv + v1 * 8]
            res = bf16_round(acc * np.float32(scale))
            for q in range(world):
                outbox[q][r * sv + v0 * 8: r * sv + v1 * 8] = res
    # (barrier) phase 3: every rank unpacks its outbox
    return [o.copy() for o in outbox]


def one_shot_allreduce(srcs: list[np.ndarray], ctas: int, scale: float) -> list[np.ndarray]:
    """Emulate ``ar_oneshot_kernel``: every rank pushes its whole bf16 buffer to every peer."""
    world = len(srcs)
    n = srcs[0].size
    nvec = n // 8
    outs = []
    wire = [bf16_round(s) for s in srcs]
    for r in range(world):
        out = np.zeros(n, np.float32)
        for _, v0, v1 in _cta_ranges(nvec, ctas):
            acc = np.zeros((v1 - v0) * 8, np.float32)
            for q in range(world):
                acc += wire[q][v0 * 8: v1 * 8]
            out[v0 * 8: v1 * 8] = acc * np.float32(scale)
        outs.append(out)
    return outs


def reduce_scatter_push(srcs: list[np.ndarray], ctas: int, scale: float) -> list[np.ndarray]:
    """Emulate ``rs_push_kernel``: rank r ends with the fp32 reduction of slice r."""
    world = len(srcs)
    n = srcs[0].size
    slice_vecs = n // 8 // world
    sv = slice_vecs * 8
    inbox = [np.zeros(n, np.float32) for _ in range(world)]
    for r in range(world):
        for _, v0, v1 in _cta_ranges(slice_vecs, ctas):
            for s in range(world):
                inbox[s][r * sv + v0 * 8: r * sv + v1 * 8] = bf16_round(srcs[r][s * sv + v0 * 8: s * sv + v1 * 8])
    shards = []
    for r in range(world):
        out = np.zeros(sv, np.float32)
        for _, v0, v1 in _cta_ranges(slice_vecs, ctas):
            acc = np.zeros((v1 - v0) * 8, np.float32)
            for q in range(world):
                acc += inbox[r][q * sv + v0 * 8: q * sv + v1 * 8]
            out[v0 * 8: v1 * 8] = acc * np.float32(scale)
        shards.append(out)
    return shards


def pipelined_allreduce(launches: list[list[np.ndarray]], ctas: int, chunk: int, scale: float,
                        seed: int = 0, epoch0: int = 1) -> list[list[np.ndarray]]:
    """Emulate ``ar_pipe_kernel`` for consecutive launches, with ranks and CTAs interleaved at random.

    Every (launch, rank, CTA) is a program of steps A(k) push / B(k) reduce / C(k) unpack in the
    kernel's order (A(k), B(k-1), C(k-2) per iteration) that waits on the same progress flags
    (slot A and slot B, value epoch * 4096 + chunks done). A scheduler repeatedly runs a random
    program whose next step is not blocked; a launch of a rank starts only after that rank's
    previous launch finished (stream order). Raises RuntimeError on a deadlock and on any read of
    an inbox / outbox cell that a different launch or chunk wrote last (a reuse race).
    Returns the fp32 outputs per launch and rank.
    """
    rnd = np.random.default_rng(seed)
    world = len(launches[0])
    n = launches[0][0].size
    slice_vecs = n // 8 // world
    sv = slice_vecs * 8
    per = (slice_vecs + ctas - 1) // ctas
    inbox = [np.zeros(n, np.float32) for _ in range(world)]
    outbox = [np.zeros(n, np.float32) for _ in range(world)]
    in_tag = [np.full(n // 8, -1, np.int64) for _ in range(world)]      # which (launch, chunk) wrote it
    out_tag = [np.full(n // 8, -1, np.int64) for _ in range(world)]
    flag_a = np.zeros((world, ctas, world), np.int64)                   # [owner][cta][src]
    flag_b = np.zeros((world, ctas, world), np.int64)
    outs = [[np.zeros(n, np.float32) for _ in range(world)] for _ in launches]

    def program(li, r, b):
        v0 = b * per
        v1 = min(v0 + per, slice_vecs)
        nch = (v1 - v0 + chunk - 1) // chunk if v1 > v0 else 0
        base = (epoch0 + li) * 4096
        steps = []
        for k in range(nch + 2):
            if k < nch:
                steps.append(("A", k))
            if 1 <= k <= nch:
                steps.append(("B", k - 1))
            if k >= 2:
                steps.append(("C", k - 2))
        return {"li": li, "r": r, "b": b, "v0": v0, "v1": v1, "base": base, "steps": steps, "pc": 0}

    def rng_of(p, k):
        c0 = p["v0"] + k * chunk
        return c0, min(c0 + chunk, p["v1"])

    def blocked(p):
        op, k = p["steps"][p["pc"]]
        want = p["base"] + k + 1
        if op == "B":
            return bool((flag_a[p["r"], p["b"], :] < want).any())
        if op == "C":
            return bool((flag_b[p["r"], p["b"], :] < want).any())
        return False

    def run(p):
        op, k = p["steps"][p["pc"]]
        li, r, b = p["li"], p["r"], p["b"]
        c0, c1 = rng_of(p, k)
        tag = li * 100000 + k
        src = launches[li][r]
        if op == "A":
            for s_ in range(world):
                seg = src[s_ * sv + c0 * 8: s_ * sv + c1 * 8]
                inbox[s_][r * sv + c0 * 8: r * sv + c1 * 8] = bf16_round(seg)
                in_tag[s_][r * slice_vecs + c0: r * slice_vecs + c1] = tag
            flag_a[:, b, r] = p["base"] + k + 1
        elif op == "B":
            acc = np.zeros((c1 - c0) * 8, np.float32)
            for q in range(world):
                if (in_tag[r][q * slice_vecs + c0: q * slice_vecs + c1] != tag).any():
                    raise RuntimeError(f"stale inbox read: launch {li} rank {r} cta {b} chunk {k} from {q}")
                acc += inbox[r][q * sv + c0 * 8: q * sv + c1 * 8]
            res = bf16_round(acc * np.float32(scale))
            for q in range(world):
                outbox[q][r * sv + c0 * 8: r * sv + c1 * 8] = res
                out_tag[q][r * slice_vecs + c0: r * slice_vecs + c1] = tag
            flag_b[:, b, r] = p["base"] + k + 1
        else:
            for s_ in range(world):
                if (out_tag[r][s_ * slice_vecs + c0: s_ * slice_vecs + c1] != tag).any():
                    raise RuntimeError(f"stale outbox read: launch {li} rank {r} cta {b} chunk {k} slice {s_}")
                outs[li][r][s_ * sv + c0 * 8: s_ * sv + c1 * 8] = outbox[r][s_ * sv + c0 * 8: s_ * sv + c1 * 8]
        p["pc"] += 1

    # per rank: the queue of launches; a rank's launch li+1 starts when all its CTAs finished li
    pending = {r: list(range(len(launches))) for r in range(world)}
    active: list[dict] = []

    def start_next(r):
        while pending[r]:
            li = pending[r].pop(0)
            progs = [pr for pr in (program(li, r, b) for b in range(ctas)) if pr["steps"]]   # empty CTAs exit
            if progs:
                active.extend(progs)
                return

    for r in range(world):
        start_next(r)
    while active:
        ready = [p for p in active if not blocked(p)]
        if not ready:
            raise RuntimeError("deadlock: every active CTA waits on a progress flag")
        p = ready[int(rnd.integers(len(ready)))]
        run(p)
        if p["pc"] == len(p["steps"]):
            active.remove(p)
            if not any(q["r"] == p["r"] and q["li"] == p["li"] for q in active):
                start_next(p["r"])
    return outs


# ------------------------------------------------------- all-gather GEMM chunk schedule
ORDER_FLAT, ORDER_OWN_FIRST, ORDER_PEERS_FIRST, ORDER_INTERLEAVED = 0, 1, 2, 3


def ag_gemm_schedule(shard_bytes: int, world: int, rank: int, lo: int, hi: int, w0: int, w_bytes: int,
                     grid: int, order: int, chunk: int = 16384) -> list[list[tuple[int, int, int]]]:
    """Per CTA, the (owner, flat start, flat end) chunks its gather lane copies, in issue order.

    Restates ``AgGate::worker`` / ``rest_chunk`` / ``owner_rest``: shard-aligned chunks clipped to
    [lo, hi); ORDER_FLAT walks all chunks from W's first one; the other orders take the chunks
    that overlap W first (flat order), then the rest by owner (own shard first, peers first, or
    interleaved chunk by chunk, starting at rank + 1).
    """
    S = shard_bytes
    cps = (S + chunk - 1) // chunk
    total = cps * world

    def chunk_of(f):
        q = f // S
        return q * cps + (f - q * S) // chunk

    wf, wl = chunk_of(w0), chunk_of(w0 + w_bytes - 1)
    cf, cl = chunk_of(lo), chunk_of(hi - 1)

    def rng(c):
        q = c // cps
        f0 = q * S + (c - q * cps) * chunk
        f1 = min(f0 + chunk, (q + 1) * S)
        return q, max(f0, lo), min(f1, hi)

    def owner_rest(q, k):
        a, b = max(q * cps, cf), min(q * cps + cps - 1, cl)
        if a > b:
            return -1
        p0a, p0b = a, min(wf - 1, b)
        p1a, p1b = max(wl + 1, a), b
        if p0b >= p0a:
            if k <= p0b - p0a:
                return p0a + k
            k -= p0b - p0a + 1
        if p1b >= p1a and k <= p1b - p1a:
            return p1a + k
        return -1

    def owner_count(q):
        a, b = max(q * cps, cf), min(q * cps + cps - 1, cl)
        if a > b:
            return 0
        ia, ib = max(a, wf), min(b, wl)
        return (b - a + 1) - (ib - ia + 1 if ib >= ia else 0)

    def rest_chunk(i):
        if order == ORDER_INTERLEAVED:
            k = i // world
            if k >= cps:
                return -2
            return owner_rest((rank + 1 + i % world) % world, k)
        for j in range(world):
            q = (rank + j + (0 if order == ORDER_OWN_FIRST else 1)) % world
            n = owner_count(q)
            if i < n:
                return owner_rest(q, i)
            i -= n
        return -2

    out = []
    for b in range(grid):
        mine = []
        if order == ORDER_FLAT:
            i = b
            while i < total:
                q, f0, f1 = rng((wf + i) % total)
                if f1 > f0:
                    mine.append((q, f0, f1))
                i += grid
        else:
            i = b
            while wf + i <= wl:
                q, f0, f1 = rng(wf + i)
                if f1 > f0:
                    mine.append((q, f0, f1))
                i += grid
            i = b
            while True:
                c = rest_chunk(i)
                i += grid
                if c == -2:
                    break
                if c < 0:
                    continue
                q, f0, f1 = rng(c)
                if f1 > f0:
                    mine.append((q, f0, f1))
        out.append(mine)
    return out
