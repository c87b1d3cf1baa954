"""Where the native attention kernels spend their cycles, phase by phase.

    python -m nuvla_forge_b200.bench.attn_phases [--shape vit|backbone] [--timeline]

Runs the tcgen05 forward and backward once each with their per-phase cycle counters switched on
(``nfb_attn_fwd_trace`` / ``nfb_attn_bwd_trace``: lane 0 of every warp adds the SM cycles spent
in each phase of its loop) and prints, per role, the average cycles per warp and per step (one
step = one 128 x 128 tile pair). Waits show which role the others stall on; the compute phases
show how far each is from its instruction or pipe bound. ``--timeline`` also prints the first
CTA's events in order (MMA batches issued per tile and step, and each softmax warp's phase
boundaries), which shows what a waiting role waits for. A profiling aid: the traced kernels are
separate instantiations, the untraced ones carry no counters.
"""

from __future__ import annotations

import argparse

import torch

FWD_PHASES = {0: "softmax: wait S", 1: "softmax: TMEM load S", 2: "softmax: row max", 3: "softmax: exp + P store",
              4: "softmax: rescale + signal", 5: "softmax: epilogue wait", 6: "softmax: epilogue store",
              8: "mma: wait P", 9: "mma: wait K/V", 10: "mma: wait PV done", 11: "mma: issue",
              16: "tma: wait slot", 17: "tma: issue"}
BWD_PHASES = {0: "compute: wait S (+Q/dO)", 1: "compute: P^T", 2: "compute: wait dQ", 3: "compute: dQ drain",
              4: "compute: wait dP", 5: "compute: dS^T", 6: "compute: final reduce wait", 7: "compute: dK/dV store",
              8: "mma: wait P^T", 9: "mma: wait Q/dO", 10: "mma: wait dV done", 11: "mma: wait dS^T",
              12: "mma: issue", 13: "mma: wait dQ drained"}

SHAPES = {"vit": (24, 1024, 1024, 16, 16, 64, False), "backbone": (2, 3392, 3392, 16, 8, 128, True)}


def _report(title, counters, phases, warps_of, ctas, steps):
    c = counters.cpu().tolist()
    print(title)
    for slot, name in phases.items():
        role = name.split(":")[0]
        if c[slot]:
            print(f"  {name:<32} {c[slot] / (warps_of[role] * ctas) / steps:10.0f} cycles/step")


def _timeline(counters, which):
    c = counters.cpu().tolist()
    ev = sorted(((v & 0xFFFFFFFFFFFF, v >> 48) for v in c[64:] if v))
    n = len(ev)
    if not ev:
        return
    t0 = ev[0][0]
    print(f"{which}: timeline of the first CTA ({n} events, SM cycles)")
    phase = ["wait S", "got S", "max done", "first-half P V done", "P ready", "first half of P stored"]
    kinds = ["S issue", "S issued", "PV(keys 0-63) issue", "PV(keys 0-63) issued", "PV(keys 64-127) issue",
             "PV(keys 64-127) issued"]
    for t, code in ev:
        if code >= 10000:
            w, rest = divmod(code - 10000, 1000)
            name = f"warp {w + 2} (tile {w // 4}) step {rest // 10}: {phase[rest % 10]}"
        elif code >= 1000:
            kind, rest = divmod(code - 1000, 100)
            name = f"    MMA tile {rest // 50} step {rest % 50}: {kinds[kind]}"
        else:
            name = str(code)
        print(f"  {t - t0:8d}  {name}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", choices=sorted(SHAPES), default="vit")
    ap.add_argument("--timeline", action="store_true", help="print the event timeline of the first CTA")
    args = ap.parse_args(argv)
    from .. import _native as nat
    from ..ops import flash_attn

    B, Sq, Sk, Hq, Hkv, D, causal = SHAPES[args.shape]
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, Sq, Hq, D, generator=g, device="cuda").to(torch.bfloat16)
    kv = torch.randn(B, Sk, 2 * Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    k, v = kv.split([Hkv, Hkv], dim=2)
    out, lse = flash_attn.attention_fwd(q, k, v, causal)
    dout = torch.randn_like(out)
    flash_attn.attention_bwd(q, k, v, out, dout, lse, causal)
    torch.cuda.synchronize()
    nq, nk = (Sq + 127) // 128, (Sk + 127) // 128
    pairs = nq * nk if not causal else sum(min(nk, i + 1) for i in range(nq))     # (query tile, key tile) pairs
    pair_heads = (Hq // Hkv) % 2 == 0
    fwd_ctas = B * (Hq // 2 * nq if pair_heads else Hq * ((Sq + 255) // 256))
    bwd_ctas = B * Hkv * nk
    G = Hq // Hkv
    for which, fn, ctas, phases, warps, steps in (
            ("forward", lambda: flash_attn.attention_fwd(q, k, v, causal), fwd_ctas, FWD_PHASES,
             {"softmax": 8, "mma": 1, "tma": 1}, pairs / nq),
            ("backward", lambda: flash_attn.attention_bwd(q, k, v, out, dout, lse, causal), bwd_ctas, BWD_PHASES,
             {"compute": 8, "mma": 1}, G * pairs / nk)):
        counters = torch.zeros(2048, dtype=torch.int64, device="cuda")
        lib = nat.lib()
        setter = lib.nfb_attn_fwd_trace if which == "forward" else lib.nfb_attn_bwd_trace
        setter(counters.data_ptr())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        setter(None)
        if args.timeline:
            _timeline(counters, which)
        c = counters.cpu().tolist()
        if which == "forward" and c[30]:
            print(f"  mma issuer poll loop: {c[31] / c[30]:.0f} cycles per iteration ({c[30] / ctas:.0f} per CTA)")
        # one step: a key tile for both query tiles of a forward CTA; a (head, query tile) for a backward CTA
        _report(f"{which} {args.shape}: {e0.elapsed_time(e1):.3f} ms (traced), {ctas} CTAs, {steps:.1f} steps each",
                counters, phases, warps, ctas, steps)
    flash_attn.check_status()


if __name__ == "__main__":
    main()
