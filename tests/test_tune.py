"""The tuner's decision logic on CPU (gemmkit-tune's rules, gemmkit-tune/src/main.rs:182-245):
the incumbent is kept unless a candidate beats it by more than the measured noise (plus 5 %
when the incumbent is "automatic"), every knob is restored after its sweep, and the profile
lists one sourceable line per knob."""
import pytest

from gemmkit_b200.tune import Stat, build_profile, geomean, sweep


def _run(default, values, spreads=None, extras=None):
    """Sweep with a fake probe that returns `values[v]` (spread in % from `spreads`)."""
    spreads = spreads or {}
    log = []

    def set_knob(name, v):
        log.append(v)

    cur = {"v": None}

    def set_and_track(name, v):
        set_knob(name, v)
        cur["v"] = v

    def probe():
        v = cur["v"]
        med, sp = values[v], spreads.get(v, 0.0)
        return Stat(med, med * (1 - sp / 200), med * (1 + sp / 200))

    extras = extras if extras is not None else [v for v in values if v != default]
    r = sweep("GEMMKIT_CUDA_X", default, extras, "u", 3, probe, set_and_track)
    return r, log


def test_incumbent_kept_without_clear_win():
    r, log = _run(1, {1: 100.0, 0: 101.0}, spreads={1: 2.0, 0: 2.0})
    assert r.winner == 1 and log == [1, 0, -1]  # tried in order, then restored
    assert r.speedup() == pytest.approx(1.0)


def test_clear_win_replaces_incumbent():
    r, _ = _run(1, {1: 100.0, 0: 110.0}, spreads={1: 2.0, 0: 2.0})
    assert r.winner == 0 and r.speedup() == pytest.approx(1.1)


def test_auto_default_needs_extra_margin():
    r, _ = _run(0, {0: 100.0, 128: 104.0, 256: 106.0})
    assert r.winner == 256  # 6 % > 5 % margin; 128's 4 % is not enough
    r, _ = _run(0, {0: 100.0, 128: 104.0})
    assert r.winner == 0


def test_duplicate_and_default_extras_are_skipped():
    r, log = _run(1, {1: 1.0, 0: 2.0}, extras=[1, 0, 0])
    assert [row.value for row in r.rows] == [1, 0] and log == [1, 0, -1]


def test_knob_restored_when_probe_fails():
    log = []

    def bad():
        raise RuntimeError("probe failed")
    with pytest.raises(RuntimeError):
        sweep("GEMMKIT_CUDA_X", 1, [0], "u", 1, bad, lambda n, v: log.append(v))
    assert log == [1, -1]


def test_geomean_and_profile_format():
    g = geomean([Stat(4.0, 3.9, 4.1), Stat(9.0, 8.0, 10.0)])
    assert g.median == pytest.approx(6.0)
    assert g.spread_pct() == pytest.approx(Stat(9.0, 8.0, 10.0).spread_pct())
    r1, _ = _run(1, {1: 100.0, 0: 120.0})
    r0, _ = _run(0, {0: 100.0, 128: 100.5})
    prof = build_profile([r1, r0], ["device test"])
    lines = [ln for ln in prof.splitlines() if ln.startswith("export ")]
    assert lines == ["export GEMMKIT_CUDA_X=0  # tuned (1.20x)",
                     "export GEMMKIT_CUDA_X=0  # default (1.00x)"]
    assert prof.startswith("# gemmkit_b200 tune profile")
