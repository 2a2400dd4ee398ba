"""gemmkit_b200.tune -- sweep the engine's knobs on this GPU and write a profile of
``export GEMMKIT_CUDA_*=...`` lines to source before running an application.

This is gemmkit-tune's method (gemmkit-tune/src/main.rs:100-245, 1578-1608) applied to the
device engine's knobs (tile width per shape class, CTA-pair kernel, its 16-warp epilogue form,
ring depth, stream-K tail, small-M streaming kernel with its even stream-K split and its
cluster K split, programmatic dependent launch), each scored on the shape class it steers:

* each knob is swept alone, every other knob at the value in effect; candidates are tried in a
  fixed order with the incumbent first;
* a candidate's score is the geometric mean, over a family of probe shapes, of the median
  throughput of `reps` timed batches (CUDA events, each batch sized to about `batch_ms`), with
  the worst per-shape spread carried along;
* a candidate replaces the incumbent only if it beats it by more than the larger of the two
  spreads (plus 5 % when the incumbent is "automatic", 0), so noise never decides a tie;
* the profile lists every knob with its winner, tagged ``tuned`` or ``default``, and the
  speed-up it measured.

Run: ``python -m gemmkit_b200.tune [--out gemmkit-cuda-tune.env] [--quick] [--dry-run]``.
"""
from __future__ import annotations

import argparse
import datetime
import math
import sys
from dataclasses import dataclass, field
from typing import Callable


@dataclass
class Stat:
    """A throughput measurement: the median with min / max of the timed batches."""
    median: float
    min: float
    max: float

    def spread_pct(self) -> float:
        return 100.0 * (self.max - self.min) / max(self.median, 1e-9)


@dataclass
class Timing:
    reps: int = 5
    batch_ms: float = 20.0


def geomean(stats: list[Stat]) -> Stat:
    """Geometric mean of the per-shape medians (each shape weighs the same), with the worst
    per-shape spread reconstructed around it."""
    n = max(len(stats), 1)
    med = math.exp(sum(math.log(max(s.median, 1e-9)) for s in stats) / n)
    spread = max((s.spread_pct() for s in stats), default=0.0)
    half = spread / 200.0
    return Stat(med, med * (1.0 - half), med * (1.0 + half))


@dataclass
class Row:
    value: int
    stat: Stat


@dataclass
class KnobResult:
    env: str
    default: int
    winner: int
    unit: str
    shapes: int
    rows: list[Row] = field(default_factory=list)

    def baseline(self) -> float:
        return self.rows[0].stat.median

    def winner_median(self) -> float:
        return next(r.stat.median for r in self.rows if r.value == self.winner)

    def speedup(self) -> float:
        return self.winner_median() / max(self.baseline(), 1e-12)


def sweep(env: str, default: int, extras: list[int], unit: str, shapes: int,
          probe: Callable[[], Stat], set_knob: Callable[[str, int], None]) -> KnobResult:
    """Try `default` then each distinct extra value of knob `env` (set through `set_knob`;
    a negative value restores the incumbent), score each with `probe`, and keep the incumbent
    unless a candidate clears it by more than the measured noise."""
    cands = [default] + [v for v in dict.fromkeys(extras) if v != default]
    rows = []
    try:
        for v in cands:
            set_knob(env, v)
            rows.append(Row(v, probe()))
    finally:
        set_knob(env, -1)
    auto_margin = 0.05 if default == 0 else 0.0
    best = 0
    for i in range(1, len(rows)):
        noise = max(rows[best].stat.spread_pct(), rows[i].stat.spread_pct()) / 100.0
        if rows[i].stat.median > rows[best].stat.median * (1.0 + noise + auto_margin):
            best = i
    return KnobResult(env, default, rows[best].value, unit, shapes, rows)


def build_profile(results: list[KnobResult], header: list[str]) -> str:
    out = ["# gemmkit_b200 tune profile. Source it before you run an application:",
           "#   source <this file>"]
    out += [f"# {h}" for h in header]
    out.append("")
    for r in results:
        tag = "default" if r.winner == r.default else "tuned"
        out.append(f"export {r.env}={r.winner}  # {tag} ({r.speedup():.2f}x)")
    out.append("")
    out.append("# measured (geomean over the probe shapes, median [min, max]):")
    for r in results:
        for row in r.rows:
            s = row.stat
            out.append(f"#   {r.env}={row.value}: {s.median:.1f} {r.unit} "
                       f"[{s.min:.1f}, {s.max:.1f}] over {r.shapes} shapes")
    return "\n".join(out) + "\n"


# ---- device probes ----------------------------------------------------------------------------

def measure(t: Timing, f: Callable[[], None], work: float) -> Stat:
    """Throughput (work per second / 1e12 or / 1e9 as the caller scales `work`) of back-to-back
    calls of `f`: three warm-up calls, one timed call to size a batch of about `t.batch_ms`, then
    `t.reps` timed batches (CUDA events on the current stream)."""
    import torch
    for _ in range(3):
        f()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    f()
    e1.record()
    torch.cuda.synchronize()
    one = max(e0.elapsed_time(e1), 1e-4)
    iters = max(1, min(20000, math.ceil(t.batch_ms / one)))
    rates = []
    for _ in range(t.reps):
        e0.record()
        for _ in range(iters):
            f()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        rates.append(work / (ms * 1e-3))
    rates.sort()
    return Stat(rates[len(rates) // 2], rates[0], rates[-1])


class TileFamily:
    """Requantized i8 GEMMs with a prepacked B (and one bf16 GEMM): the tile kernels' shapes.
    Rate in TOPS / TFLOP/s."""

    def __init__(self, quick: bool):
        import torch

        import gemmkit_b200 as gk
        self.gk = gk
        g = torch.Generator(device="cuda").manual_seed(11)
        shapes = ([(2048, 2048, 2048), (1000, 1000, 1000)] if quick else
                  [(4096, 4096, 4096), (2048, 4096, 1024), (1000, 1000, 1000),
                   (3072, 2048, 2304), (700, 2000, 300)])
        self.calls = []
        for m, k, n in shapes:
            a = torch.randint(-127, 128, (m * k,), dtype=torch.int8, device="cuda", generator=g)
            bT = torch.randint(-127, 128, (n * k,), dtype=torch.int8, device="cuda", generator=g)
            sc = (torch.rand(n, device="cuda", generator=g) * 9e-4 + 1e-4).float()
            packed = gk.prepack_rhs_i8(gk.MatRef.new(bT, k, n, 1, k))
            c = torch.empty(m * n, dtype=torch.int8, device="cuda")
            req = gk.Requantize(gk.RequantScale.PerCol(sc), 0)
            keep = (a, bT, sc, packed, c, req)

            def call(m=m, k=k, n=n, keep=keep):
                a, _, _, packed, c, req = keep
                gk.gemm_i8_packed_b_requant(m, a.data_ptr(), k, 1, packed, req, c.data_ptr(),
                                            1, m)
            self.calls.append((call, 2.0 * m * n * k / 1e12, keep))
        # row-major A and B -> i32 (B read MN-major, or packed K-major)
        r = 1024
        ra = torch.randint(-128, 128, (r * r,), dtype=torch.int8, device="cuda", generator=g)
        rb = torch.randint(-128, 128, (r * r,), dtype=torch.int8, device="cuda", generator=g)
        rc = torch.empty(r * r, dtype=torch.int32, device="cuda")

        def rcall(r=r, keep=(ra, rb, rc)):
            ra, rb, rc = keep
            gk.gemm_i8_unchecked(r, r, r, 1, ra.data_ptr(), r, 1, rb.data_ptr(), r, 1, 0,
                                 rc.data_ptr(), r, 1)
        self.calls.append((rcall, 2.0 * r ** 3 / 1e12, (ra, rb, rc)))
        s = 2048 if quick else 4096
        ha = torch.randn(s * s, device="cuda", generator=g).to(torch.bfloat16)
        hb = torch.randn(s * s, device="cuda", generator=g).to(torch.bfloat16)
        hc = torch.empty(s * s, device="cuda")

        def hcall(s=s, keep=(ha, hb, hc)):
            ha, hb, hc = keep
            gk.gemm_bf16_f32_unchecked(s, s, s, 1.0, ha.data_ptr(), s, 1, hb.data_ptr(), 1, s,
                                       0.0, hc.data_ptr(), s, 1)
        self.calls.append((hcall, 2.0 * s ** 3 / 1e12, (ha, hb, hc)))
        self.unit = "T(FL)OP/s"

    def probe(self, t: Timing) -> Stat:
        return geomean([measure(t, f, w) for f, w, _ in self.calls])


class ShortKFamily:
    """Products whose K is one or two 128-byte blocks, where the requantizing epilogue is the
    kernel: a batched requantized GEMM of BASELINE config 4's element shape and one plain
    requantized GEMM with K = 200. Rate in GB/s of algorithmic traffic."""

    def __init__(self, quick: bool):
        import torch

        import gemmkit_b200 as gk
        g = torch.Generator(device="cuda").manual_seed(13)
        self.calls = []
        B, m, n, k = (64 if quick else 256), 512, 512, 128
        a = torch.randint(-128, 128, (B * m * k,), dtype=torch.int8, device="cuda", generator=g)
        bT = torch.randint(-128, 128, (B * n * k,), dtype=torch.int8, device="cuda", generator=g)
        bias = torch.randint(-2**15, 2**15 + 1, (B * m,), dtype=torch.int32, device="cuda",
                             generator=g)
        sc = (torch.rand(B * n, device="cuda", generator=g) * 9e-4 + 1e-4).float()
        c = torch.empty(B * m * n, dtype=torch.uint8, device="cuda")
        req = gk.Requantize(gk.RequantScale.PerCol(sc), 128, bias, gk.AXIS_ROW)
        keep = (a, bT, bias, sc, c, req)

        def bcall(keep=keep):
            a, bT, _, _, c, req = keep
            gk.gemm_i8_requant_batched(B, m, k, n, a.data_ptr(), k, 1, m * k, bT.data_ptr(), 1, k,
                                       n * k, req, m, n, c.data_ptr(), 1, m, m * n, out_u8=True)
        self.calls.append((bcall, B * (m * k + n * k + m * n + 4 * m + 4 * n) / 1e9, keep))
        m2, k2, n2 = (2048, 200, 2048) if quick else (4096, 200, 4096)
        a2 = torch.randint(-127, 128, (m2 * k2,), dtype=torch.int8, device="cuda", generator=g)
        b2 = torch.randint(-127, 128, (n2 * k2,), dtype=torch.int8, device="cuda", generator=g)
        sc2 = (torch.rand(n2, device="cuda", generator=g) * 9e-4 + 1e-4).float()
        c2 = torch.empty(m2 * n2, dtype=torch.int8, device="cuda")
        req2 = gk.Requantize(gk.RequantScale.PerCol(sc2), 0)
        keep2 = (a2, b2, sc2, c2, req2)

        def kcall(keep=keep2):
            a2, b2, _, c2, req2 = keep
            gk.gemm_i8_requant_ex_unchecked(m2, k2, n2, a2.data_ptr(), k2, 1, b2.data_ptr(), 1,
                                            k2, req2, c2.data_ptr(), 1, m2)
        self.calls.append((kcall, (m2 * k2 + n2 * k2 + m2 * n2 + 4 * n2) / 1e9, keep2))
        self.unit = "GB/s"

    def probe(self, t: Timing) -> Stat:
        return geomean([measure(t, f, w) for f, w, _ in self.calls])


class SmallMFamily:
    """Back-to-back requantized small-M calls over prepacked weights (BASELINE config 5 shapes),
    so launch overlap counts. Rate in GB/s of weight streaming."""

    def __init__(self, quick: bool):
        import torch

        import gemmkit_b200 as gk
        g = torch.Generator(device="cuda").manual_seed(12)
        k, n = 4096, (7168 if quick else 14336)
        self.calls = []
        sets = []
        # a narrow weight matrix too (few 128-channel tiles: the cluster K split)
        bTn = torch.randint(-127, 128, (2048 * k,), dtype=torch.int8, device="cuda", generator=g)
        scn = (torch.rand(2048, device="cuda", generator=g) * 9e-4 + 1e-4).float()
        narrow = (gk.prepack_rhs_i8(gk.MatRef.new(bTn, k, 2048, 1, k)), scn)
        del bTn
        an = torch.randint(-127, 128, (k,), dtype=torch.int8, device="cuda", generator=g)
        cn = torch.empty(2048, dtype=torch.int8, device="cuda")
        reqn = gk.Requantize(gk.RequantScale.PerCol(scn), 0)

        def ncall(keep=(an, cn, narrow, reqn)):
            an, cn, narrow, reqn = keep
            gk.gemm_i8_packed_b_requant(1, an.data_ptr(), k, 1, narrow[0], reqn, cn.data_ptr(),
                                        2048, 1)
        self.calls.append((ncall, (k * 2048 + k + 2048 + 4 * 2048) / 1e9, (an, cn, narrow, reqn)))
        for _ in range(3):  # rotate weight sets so the stream does not sit in L2
            bT = torch.randint(-127, 128, (n * k,), dtype=torch.int8, device="cuda", generator=g)
            sc = (torch.rand(n, device="cuda", generator=g) * 9e-4 + 1e-4).float()
            sets.append((gk.prepack_rhs_i8(gk.MatRef.new(bT, k, n, 1, k)), sc))
            del bT
        for M in ((1, 16) if quick else (1, 4, 16)):
            a = torch.randint(-127, 128, (M * k,), dtype=torch.int8, device="cuda", generator=g)
            c = torch.empty(M * n, dtype=torch.int8, device="cuda")
            reqs = [gk.Requantize(gk.RequantScale.PerCol(sc), 0) for _, sc in sets]
            keep = (a, c, sets, reqs)

            def call(M=M, keep=keep, state=[0]):
                a, c, sets, reqs = keep
                i = state[0] % len(sets)
                state[0] += 1
                gk.gemm_i8_packed_b_requant(M, a.data_ptr(), k, 1, sets[i][0], reqs[i],
                                            c.data_ptr(), n, 1)
            self.calls.append((call, (k * n + M * k + M * n + 4 * n) / 1e9, keep))
        self.unit = "GB/s"

    def probe(self, t: Timing) -> Stat:
        return geomean([measure(t, f, w) for f, w, _ in self.calls])


# knob -> (extra candidates, families it is scored on). The families are gemmkit-tune's shape
# classes for this engine: large tiles, short K (epilogue-bound) and small M (bandwidth-bound);
# the tile width gets one entry per class (GEMMKIT_CUDA_BN, GEMMKIT_CUDA_BN_SHORTK).
KNOBS = {
    "GEMMKIT_CUDA_BN": ([128, 192, 256], ("tile",)),
    "GEMMKIT_CUDA_PAIR": ([0, 1], ("tile",)),
    "GEMMKIT_CUDA_STREAMK": ([0, 1], ("tile",)),
    "GEMMKIT_CUDA_STAGES": ([4, 6, 8], ("tile", "short_k")),
    "GEMMKIT_CUDA_BN_SHORTK": ([128, 256], ("short_k",)),
    "GEMMKIT_CUDA_EPI16": ([0, 1], ("short_k",)),
    "GEMMKIT_CUDA_GEMV": ([0, 1], ("small_m",)),
    "GEMMKIT_CUDA_GEMV_SK": ([0, 1], ("small_m",)),
    "GEMMKIT_CUDA_GEMV_SPLIT": ([2, 4, 8], ("small_m",)),
    "GEMMKIT_CUDA_PDL": ([0, 1], ("small_m", "tile")),
    "GEMMKIT_CUDA_MN_B": ([0, 1], ("tile",)),
    "GEMMKIT_CUDA_REQUANT_F32": ([0, 1], ("short_k",)),
}


def run(argv=None) -> tuple[list[KnobResult], str]:
    ap = argparse.ArgumentParser(prog="python -m gemmkit_b200.tune", description=__doc__.split(
        "\n\n")[0], formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", default="gemmkit-cuda-tune.env", help="profile path")
    ap.add_argument("--dry-run", action="store_true", help="print the report, write no profile")
    ap.add_argument("--quick", action="store_true", help="fewer, smaller probe shapes")
    ap.add_argument("--reps", type=int, default=None, help="timed batches per measurement")
    ap.add_argument("--batch-ms", type=float, default=None, help="length of one timed batch")
    ap.add_argument("--knobs", default=",".join(KNOBS), help="comma-separated knobs to sweep")
    args = ap.parse_args(argv)

    import torch

    import gemmkit_b200 as gk
    t = Timing(reps=args.reps or (3 if args.quick else 5),
               batch_ms=args.batch_ms or (5.0 if args.quick else 20.0))
    names = [k for k in args.knobs.split(",") if k]
    for k in names:
        if k not in KNOBS:
            raise SystemExit(f"unknown knob {k}; known: {', '.join(KNOBS)}")
    need = {f for k in names for f in KNOBS[k][1]}
    fams = {}
    if "tile" in need:
        fams["tile"] = TileFamily(args.quick)
    if "short_k" in need:
        fams["short_k"] = ShortKFamily(args.quick)
    if "small_m" in need:
        fams["small_m"] = SmallMFamily(args.quick)

    results = []
    for k in names:
        extras, fam_names = KNOBS[k]
        incumbent = gk.knob_get(k)

        def probe(fam_names=fam_names):
            return geomean([fams[f].probe(t) for f in fam_names])
        units = "+".join(fams[f].unit for f in fam_names)
        shapes = sum(len(fams[f].calls) for f in fam_names)
        r = sweep(k, incumbent, extras, units, shapes, probe, gk.knob_set)
        results.append(r)
        print(f"{k}: " + ", ".join(f"{row.value} -> {row.stat.median:.1f}" for row in r.rows) +
              f"  => {r.winner} ({r.speedup():.2f}x)", flush=True)

    prop = torch.cuda.get_device_properties(0)
    header = [f"generated {datetime.datetime.now(datetime.timezone.utc).isoformat(timespec='seconds')}",
              f"device {prop.name}, {prop.multi_processor_count} SMs, torch {torch.__version__}, "
              f"CUDA {torch.version.cuda}",
              f"timing: {t.reps} batches of ~{t.batch_ms} ms per measurement"
              + (", quick shapes" if args.quick else "")]
    profile = build_profile(results, header)
    if args.dry_run:
        print(profile)
    else:
        with open(args.out, "w") as f:
            f.write(profile)
        print(f"profile written to {args.out}")
    return results, profile


def main(argv=None) -> int:
    run(argv)
    return 0


if __name__ == "__main__":
    sys.exit(main())
