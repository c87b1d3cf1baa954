"""Turn reports/*.json into RESULTS.md.

    python -m nuvla_forge_b200.bench.report [--reports reports] [--out RESULTS.md]

Parity: nuvla_forge/bench/report.py — it only formats what the benchmarks
wrote, cannot invent a number, and prints "_Not run._" for a missing report.
Lower-is-better rows are labelled as such (the reference labelled its peak
memory row "faster").
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path


def _load(d: Path, name: str):
    p = d / name
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except json.JSONDecodeError:
        return None


def fmt(v, spec=".2f", missing="—"):
    if v is None:
        return missing
    try:
        return format(v, spec)
    except (TypeError, ValueError):
        return str(v)


def section_kernels(lines, k):
    lines += ["## Kernel microbenchmarks", ""]
    if not k:
        lines += ["_Not run._", ""]
        return
    pk = k.get("peaks", {})
    lines += [f"Device `{k.get('device')}`; measured peaks {fmt(pk.get('hbm_gbs'), '.0f')} GB/s, "
              f"{fmt(pk.get('bf16_tflops'), '.0f')} TFLOP/s ({pk.get('source')}). Reference Triton timed: "
              f"{k.get('reference_triton')}.", ""]
    for key, title in (("adaln", "Fused adaLN-Zero + gated residual + RMSNorm (fwd+bwd)"), ("swiglu", "SwiGLU (fwd+bwd)")):
        lines += [f"### {title}", "", "| shape | eager ms | reference Triton ms | native ms | vs Triton | achieved GB/s | of measured HBM |",
                  "|---|---|---|---|---|---|---|"]
        for r in k.get(key, []):
            lines.append(f"| `{r['shape']}` | {fmt(r.get('eager_ms'), '.3f')} | {fmt(r.get('reference_triton_ms'), '.3f')} | "
                         f"{fmt(r.get('native_ms'), '.3f')} | {fmt(r.get('speedup_vs_reference_triton'))}x | "
                         f"{fmt(r.get('achieved_gb_s'), '.0f')} | {fmt(100 * r.get('frac_of_measured_hbm', 0), '.0f')}% |")
        lines.append("")
        timed = [r for r in k.get(key, []) if r.get("native_fwd_kernel_ms")]
        if timed:
            lines += ["The two native kernels alone (L2 flushed before each; the table above times forward, "
                      "autograd and backward back to back):", ""]
            for r in timed:
                lines.append(f"* `{r['shape']}`: forward {fmt(r['native_fwd_kernel_ms'], '.3f')} ms + backward "
                             f"{fmt(r['native_bwd_kernel_ms'], '.3f')} ms = {fmt(r.get('kernels_gb_s'), '.0f')} GB/s, "
                             f"{fmt(100 * r.get('kernels_frac_of_measured_hbm', 0), '.0f')}% of measured HBM")
            lines.append("")
    if k.get("patchify"):
        lines += ["### Patchify (uint8 HWC frames -> normalised bf16 patch rows)", "",
                  "| shape | eager ms | native ms | vs eager | achieved GB/s | of measured HBM |", "|---|---|---|---|---|---|"]
        for r in k["patchify"]:
            lines.append(f"| `{r['shape']}` | {fmt(r.get('eager_ms'), '.3f')} | {fmt(r.get('native_ms'), '.3f')} | "
                         f"{fmt(r.get('speedup_vs_eager'))}x | {fmt(r.get('achieved_gb_s'), '.0f')} | "
                         f"{fmt(100 * r.get('frac_of_measured_hbm', 0), '.0f')}% |")
        lines.append("")
    lines += ["### Cross entropy (fwd+bwd; peak memory: lower is better)", "",
              "| shape | naive ms / MiB | reference Triton ms / MiB | native ms / MiB | vs Triton | TFLOP/s (3 GEMMs) |",
              "|---|---|---|---|---|---|"]
    for r in k.get("cross_entropy", []):
        lines.append(f"| `{r['shape']}` | {fmt(r.get('naive_ms'))} / {fmt(r.get('naive_peak_mib'), '.0f')} | "
                     f"{fmt(r.get('reference_triton_ms'))} / {fmt(r.get('reference_triton_peak_mib'), '.0f')} | "
                     f"{fmt(r.get('native_ms'))} / {fmt(r.get('native_peak_mib'), '.0f')} | "
                     f"{fmt(r.get('speedup_vs_reference_triton'))}x | {fmt(r.get('achieved_tflops'), '.0f')} |")
    lines.append("")


def section_comms(lines, reports: Path):
    lines += ["## Collectives (bus GB/s, fused vs NCCL)", ""]
    found = sorted(reports.glob("comms*.json"))
    if not found:
        lines += ["_Not run._", ""]
        return
    for p in found:
        c = json.loads(p.read_text())
        lines += [f"### {p.name}: world {c['world_size']}, NCCL {c.get('nccl_version')}", "",
                  "| bytes | CTAs | AR fused | AR pipelined | AR NCCL bf16 | AR NCCL fp32 | RS fused | RS NCCL | AG fused | "
                  "AG NCCL |", "|---|---|---|---|---|---|---|---|---|---|"]
        for r in c["rows"]:
            lines.append(f"| {r['bytes']} | {r.get('ctas', '—')} | {fmt(r['ar_fused_busbw'], '.1f')} | "
                         f"{fmt(r.get('ar_fused_pipelined_busbw'), '.1f')} | {fmt(r['ar_nccl_bf16_busbw'], '.1f')} | "
                         f"{fmt(r['ar_nccl_fp32_busbw'], '.1f')} | {fmt(r['rs_fused_busbw'], '.1f')} | "
                         f"{fmt(r['rs_nccl_busbw'], '.1f')} | {fmt(r['ag_fused_busbw'], '.1f')} | "
                         f"{fmt(r['ag_nccl_busbw'], '.1f')} |")
        lines.append("")


def section_train(lines, reports: Path):
    lines += ["## Training step", ""]
    found = sorted(reports.glob("train-*.json")) + sorted(reports.glob("bench*.json"))
    if not found:
        lines += ["_Not run._", ""]
        return
    lines += ["| report | samples/s | ms/step | world | global batch | peak MiB |", "|---|---|---|---|---|---|"]
    for p in found:
        r = json.loads(p.read_text())
        sps = r.get("samples_per_sec_max_over_ranks", r.get("samples_per_sec", r.get("value")))
        lines.append(f"| {p.name} | {fmt(sps, '.2f')} | {fmt(r.get('step_ms', r.get('ms_per_step')), '.1f')} | "
                     f"{r.get('world_size', r.get('n_gpus'))} | {r.get('global_batch', r.get('config', {}).get('global_batch'))} | "
                     f"{fmt(r.get('peak_mem_mib'), '.0f')} |")
    lines.append("")


def section_ag_gemm(lines, reports: Path):
    lines += ["## All-gather fused into the first consuming GEMM", ""]
    found = sorted(reports.glob("ag_gemm_n*.json"))
    if not found:
        lines += ["_Not run._", ""]
        return
    lines += ["| GPUs | unit -> GEMM | fused ms | hybrid ms | separate ms | copy-engine + GEMM ms | roofline ms | "
              "fused fraction of roofline |", "|---|---|---|---|---|---|---|---|"]
    for p in found:
        d = json.loads(p.read_text())
        for r in d["rows"]:
            lines.append(f"| {d['world_size']} | {r['case']} | {fmt(r.get('fused_ms'), '.3f')} | "
                         f"{fmt(r.get('fused_w_ce_ms'), '.3f')} | {fmt(r.get('separate_ms'), '.3f')} | "
                         f"{fmt(r.get('separate_ce_ms'), '.3f')} | {fmt(r.get('roofline_ms'), '.3f')} "
                         f"({r.get('roofline_bound')}) | {fmt(100 * r['frac_of_roofline'], '.0f')}% |")
    lines.append("")


def section_attention(lines, d):
    lines += ["## Attention forward and backward (tcgen05 kernels vs PyTorch SDPA / cuDNN)", ""]
    if not d:
        lines += ["_Not run._", ""]
        return
    lines += ["| shape | fwd native ms (TFLOP/s) | fwd SDPA ms (TFLOP/s) | bwd native ms (TFLOP/s) | "
              "bwd SDPA ms (TFLOP/s) |", "|---|---|---|---|---|"]
    for r in d["rows"]:
        lines.append(f"| {r['shape']} | {fmt(r['native_ms'], '.3f')} ({fmt(r['native_tflops'], '.0f')}) | "
                     f"{fmt(r['sdpa_ms'], '.3f')} ({fmt(r['sdpa_tflops'], '.0f')}) | "
                     f"{fmt(r.get('native_bwd_ms'), '.3f')} ({fmt(r.get('native_bwd_tflops'), '.0f')}) | "
                     f"{fmt(r.get('sdpa_bwd_ms'), '.3f')} ({fmt(r.get('sdpa_bwd_tflops'), '.0f')}) |")
    lines.append("")


def section_mma_rates(lines, d):
    lines += ["## tcgen05.mma throughput by shape and operand source (bench_mma_rates)", ""]
    if not d:
        lines += ["_Not run._", ""]
        return
    lines += ["| instruction | operands | cycles / instruction | FLOP / clk / SM | of 8192 |", "|---|---|---|---|---|"]
    for r in d["rows"]:
        lines.append(f"| M128 N{r['n']} K16 | {r['operands']} | {fmt(r['cycles_per_instr'], '.1f')} | "
                     f"{fmt(r['flop_per_clk_per_sm'], '.0f')} | {fmt(100 * r['frac_of_8192'], '.0f')}% |")
    lines.append("")


def section_gemm(lines, d, sus):
    lines += ["## Linear-layer GEMMs (CTA-pair tcgen05 kernel vs cuBLAS)", ""]
    if not d:
        lines += ["_Not run._", ""]
    else:
        pk = (d.get("measured_peaks") or {}).get("bf16_tflops")
        lines += [f"Burst, L2 flushed between iterations; measured cuBLAS bf16 peak {fmt(pk, '.0f')} TFLOP/s.", "",
                  "| shape (M x N x K) | role | native ms | native TFLOP/s | cuBLAS ms | cuBLAS TFLOP/s | speed-up |",
                  "|---|---|---|---|---|---|---|"]
        for r in d["rows"]:
            lines.append(f"| {r['shape']} {r['M']}x{r['N']}x{r['K']} | {r['role']} | {fmt(r['native_ms'], '.3f')} | "
                         f"{fmt(r['native_tflops'], '.0f')} | {fmt(r['cublas_ms'], '.3f')} | "
                         f"{fmt(r['cublas_tflops'], '.0f')} | {fmt(r['speedup'], '.3f')}x |")
        lines.append("")
    if sus:
        lines += [f"Sustained ({sus['sustained_s']} s back to back per case, under the 1 kW power cap):", "",
                  "| shape | role | impl | TFLOP/s | SM MHz | W | pJ/FLOP |", "|---|---|---|---|---|---|---|"]
        for r in sus["rows"]:
            c = r.get("clocks") or {}
            lines.append(f"| {r['shape']} | {r.get('role', 'fwd')} | {r['impl']} | {fmt(r['tflops'], '.0f')} | "
                         f"{fmt(c.get('sm_mhz'), '.0f')} | {fmt(c.get('power_w'), '.0f')} | "
                         f"{fmt(r.get('pj_per_flop'), '.3f')} |")
        lines.append("")


def section_planner(lines, d):
    lines += ["## Planning latency (DiT sampling loop, eager vs CUDA graph)", ""]
    if not d:
        lines += ["_Not run._", ""]
        return
    lines += [f"Model `{d['model']}`, {d['steps']} Euler steps.", "", "| batch | eager ms | graphed ms | speed-up |",
              "|---|---|---|---|"]
    for r in d["rows"]:
        lines.append(f"| {r['batch']} | {fmt(r['eager_ms'])} | {fmt(r['graphed_ms'])} | {fmt(r['speedup'])}x |")
    lines.append("")


def section_loader(lines, d):
    lines += ["## Data loading", ""]
    if not d:
        lines += ["_Not run._", ""]
        return
    lines += ["| config | samples/s | GPU idle |", "|---|---|---|"]
    for r in d.get("configs", []):
        lines.append(f"| {r['config']} | {fmt(r.get('samples_per_sec'), '.1f')} | {fmt(r.get('gpu_idle_pct'), '.1f')}% |")
    lines.append("")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reports", default="reports")
    ap.add_argument("--out", default="RESULTS.md")
    args = ap.parse_args(argv)
    d = Path(args.reports)
    lines = ["# RESULTS", "", "Generated by `python -m nuvla_forge_b200.bench.report` from `reports/*.json`.", ""]
    hw = d / "hardware.txt"
    lines += ["## Hardware", ""] + (["```", hw.read_text().strip()[:3000], "```", ""] if hw.exists() else
                                    ["_Not captured (python -m nuvla_forge_b200.utils.probe)._", ""])
    section_train(lines, d)
    section_kernels(lines, _load(d, "kernels.json"))
    section_comms(lines, d)
    section_ag_gemm(lines, d)
    section_gemm(lines, _load(d, "gemm.json"), _load(d, "gemm_sustained.json"))
    section_attention(lines, _load(d, "attention.json"))
    section_mma_rates(lines, _load(d, "mma_rates.json"))
    section_planner(lines, _load(d, "planner.json"))
    section_loader(lines, _load(d, "dataloader.json"))
    Path(args.out).write_text("\n".join(lines) + "\n")
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
