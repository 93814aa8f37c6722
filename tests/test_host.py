"""Host-side logic (no GPU): geometry, weights, conversion, FLOP accounting, and the
C ABI library's exports."""
import ctypes
import subprocess

import numpy as np
import pytest

from s2s_testlib import ROOT, pkg


def test_plan_pads_to_next_window_multiple():
    P = pkg()
    # src/plan.rs:39-47: an exact multiple still gains a whole window.
    pl = P.plan.Plan.new(1080, 1920, 8, 180)
    assert (pl.hp, pl.wp) == (1088, 1928)
    pl = P.plan.Plan.new(240, 320, 8, 180)
    assert (pl.hp, pl.wp, pl.nw, pl.tokens()) == (248, 328, 31 * 41, 81344)


def test_plan_index_and_region_follow_the_rolled_plane():
    P = pkg()
    pl = P.plan.Plan.new(16, 24, 8, 1)          # 24 x 32 plane, 3 x 4 windows
    # shifted block: token (0,0) of window 0 reads (4, 4)
    assert pl.index(0, 0, 4) == (4, 4)
    # the last window row wraps to image row 0..3
    assert pl.index(2 * pl.nww, 7 * 8, 4)[0] == (16 + 7 + 4) % 24
    # regions on the unwrapped coordinate (src/plan.rs:84-108)
    assert pl.region(0, 0, 4) == (0, 0)
    last = pl.nw - 1
    assert pl.region(last, 63, 4) == (2, 2)
    assert pl.region(last, 0, 4) == (1, 1)
    # token_pixels is the vectorised index()
    tp = pl.token_pixels(4)
    for wi, t in [(0, 0), (5, 17), (last, 63)]:
        y, x = pl.index(wi, t, 4)
        assert tp[wi * 64 + t] == y * pl.wp + x
    assert sorted(tp.tolist()) == list(range(pl.plane()))


def test_too_small_image_is_refused():
    P = pkg()
    with pytest.raises(ValueError, match="smaller than one 8x8 window"):
        P.plan.check_size(7, 64, 8)


def test_seeded_weights_are_deterministic_and_validated():
    P = pkg()
    a = P.weights.Weights.seeded("lightweight_sr", 0)
    b = P.weights.Weights.seeded("lightweight_sr", 0)
    for k in a.tensors:
        assert np.array_equal(a.t(k), b.t(k)), k
    assert a.upsampler == "pixelshuffledirect" and a.depths == [6, 6, 6, 6]
    assert a.t("layers.0.residual_group.blocks.0.attn.cpb_pre").shape == (4096, 6)
    # linear init is normal(0, .02) clamped to two std
    w = a.t("layers.0.residual_group.blocks.0.mlp.fc1.weight")
    assert np.abs(w).max() <= 0.04 + 1e-7 and 0.015 < w.std() < 0.02


def test_convert_slices_qkv_and_builds_cpb_table():
    P = pkg()
    sd = P.weights.seeded_state_dict("lightweight_sr", 3, perturb=True)
    t, meta = P.weights.convert(sd, "lightweight_sr")
    p = "layers.1.residual_group.blocks.2.attn"
    q = sd[f"{p}.qkv.weight"]
    assert np.array_equal(t[f"{p}.qkv.wk"], q[60:120])
    assert meta["upsampler"] == "pixelshuffledirect" and meta["depths"] == "6,6,6,6"
    cpb = t[f"{p}.cpb_pre"]
    assert cpb.shape == (4096, 6) and cpb.min() > 0 and cpb.max() < 16


def test_safetensors_roundtrip_and_tamper(tmp_path):
    P = pkg()
    wt = P.weights.Weights.seeded("lightweight_sr", 0)
    path = tmp_path / "lw.safetensors"
    P.weights.save_safetensors(path, wt.tensors, wt.meta)
    back = P.weights.Weights.load(path)
    assert back.depths == wt.depths
    for k in wt.tensors:
        assert np.array_equal(back.t(k), wt.t(k))
    # a header promising a missing stage is refused, naming the tensor
    # (tests/parity.rs:198-224 of the reference)
    meta = dict(wt.meta, depths="6,6,6,6,6")
    with pytest.raises(ValueError, match="layers.4.residual_group.blocks.0"):
        P.weights.Weights(wt.tensors, meta)


def test_flops_match_the_algorithmic_accounting():
    P = pkg()
    wt = P.weights.Weights.seeded("classical_sr", 0)
    f = wt.flops_forward(248, 328)
    assert abs(f / 1e9 - 2164) < 2            # 2 164 GFLOP for classical-x4 240x320
    lw = P.weights.Weights.seeded("lightweight_sr", 0)
    assert abs(lw.flops_forward(72, 72) / 1e9 - 11.0) < 0.1


def _lib_path():
    import importlib
    pkg()
    capi = importlib.import_module("swin2sr_b200.capi")
    if not capi.LIB_PATH.exists():
        importlib.import_module("swin2sr_b200.build").build()
    return capi.LIB_PATH


def test_c_abi_library_exports_every_declared_symbol():
    import importlib
    P = pkg()
    capi = importlib.import_module("swin2sr_b200.capi")
    path = _lib_path()
    header = (ROOT / "include" / "s2s.h").read_text()
    import re
    declared = set(re.findall(r"\b(s2s_[a-z0-9_]+)\s*\(", header))
    assert declared == set(capi.EXPORTS), declared ^ set(capi.EXPORTS)
    lib = ctypes.CDLL(str(path))            # loads without a GPU: no CUDA call at load time
    for sym in declared:
        assert hasattr(lib, sym), sym
    lib.s2s_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.s2s_version()
    nm = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True,
                        text=True).stdout
    for sym in declared:
        assert f" T {sym}" in nm, sym


def test_library_refuses_bad_config_without_touching_the_device():
    import importlib
    capi = importlib.import_module("swin2sr_b200.capi")
    _lib_path()
    L = capi.load()
    cfg = capi.S2SConfig()
    cfg.window = 7                           # unsupported: rejected before any CUDA call
    h = ctypes.c_void_p()
    rc = L.s2s_create(ctypes.byref(cfg), None, 0, 0, ctypes.byref(h))
    assert rc == capi.S2S_ERR_UNSUPPORTED and not h.value
    assert b"unsupported" in L.s2s_last_error(None)


def test_workloads_are_seeded_and_in_range():
    import importlib
    wl = importlib.import_module("swin2sr_b200.workloads")
    a = wl.make_input("classical-x4")
    b = wl.make_input("classical-x4")
    assert a.shape == (1, 3, 240, 320) and np.array_equal(a, b)
    assert 0.0 <= a.min() and a.max() <= 1.0 and a.std() > 0.05
    rw = wl.make_input("realworld-x4")
    assert rw.shape == (1, 3, 512, 512) and 0.0 <= rw.min() and rw.max() <= 1.0


def test_gelu_erf_approximation_bound():
    """The kernels' GELU uses Abramowitz & Stegun 7.1.28 for erf (csrc/common.cuh,
    gelu_erf); evaluated in fp32 with the same operation order it stays within 1e-6
    absolute of the exact erf-form GELU the reference computes (src/cpu.rs:1125-1132)."""
    import math
    a = np.array([0.0705230784, 0.0422820123, 0.0092705272, 0.0001520143, 0.0002765672,
                  0.0000430638], np.float32)
    x = np.linspace(-12, 12, 200001).astype(np.float32)
    t = np.abs(x) * np.float32(0.70710678118654752440)
    p = a[5]
    for c in a[4::-1]:
        p = p * t + c
    p = p * t + np.float32(1.0)
    for _ in range(4):
        p = p * p
    h = np.float32(0.5) * x * (np.float32(1.0) / p)
    got = np.where(x >= 0, x - h, h).astype(np.float64)
    ref = np.array([0.5 * float(v) * (1 + math.erf(float(v) / math.sqrt(2))) for v in x])
    assert np.abs(got - ref).max() < 1e-6


def test_bench_kernel_accounting_adds_up_to_the_forward():
    """bench.py's per-launch FLOPs of each kernel class (the roofline's numerator),
    summed over one classical-x4 forward's launches, equal the model's algorithmic
    FLOPs; the MLP's algorithmic bytes are 12 bytes per padded channel per token."""
    import importlib.util
    P = pkg()
    spec = importlib.util.spec_from_file_location("s2s_bench", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    wt = P.weights.Weights.seeded("classical_sr", 0)
    hp, wp = 248, 328
    f = bench.kernel_flops(wt, 1, hp, wp)
    blocks, stages = sum(wt.depths), len(wt.depths)
    per_forward = {"qkv_attention": blocks, "proj_mlp": blocks, "conv_stage": stages, "gemm_stage_pe": stages,
                   "gemm_patch_embed": 1, "conv_after_body": 1, "conv_first": 1,
                   "conv_before_upsample": 1, "conv_upsample0": 1, "conv_upsample1": 1,
                   "conv_last": 1}
    total = sum(f[k] * n for k, n in per_forward.items())
    assert total == wt.flops_forward(hp, wp)
    # the fused MLP counts fc1 + fc2, the unfused classes the same work split in two
    assert f["mlp_fused"] == f["gemm_fc1"] + f["gemm_fc2"]
    # the fused QKV + attention kernel counts what the QKV GEMM and attention kernel do
    assert f["qkv_attention"] == f["gemm_qkv"] + f["window_attention"]
    assert f["proj_mlp"] == f["gemm_proj"] + f["mlp_fused"]
    T, Cp = hp * wp, 192
    assert bench.kernel_bytes(wt, 1, hp, wp)["mlp_fused"] == T * Cp * 12


def test_bench_clock_sampler_reports_median_clock_and_throttle_reasons():
    """The clocks record beside every bench number: median SM clock under load, the
    maximum, and every throttle reason seen active in any sample."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("s2s_bench2", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)

    class FakeProc:
        def __init__(self, text):
            self.text = text

        def terminate(self):
            pass

        def communicate(self, timeout=None):
            return self.text, ""

    rows = [
        "0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1920, 1965, 980.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 990.5, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
        "0, [N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    cs = bench.ClockSampler(0)
    cs.proc = FakeProc("\n".join(rows))
    rec = cs.stop()
    assert rec == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3}
    cs.proc = FakeProc("0, 1200, 1965, 500, 0x40, Active, Not Active, Active, Not Active\n")
    rec = cs.stop()
    assert rec["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"] and rec["sm_mhz"] == 1200.0
    cs.proc = None
    assert cs.stop() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_selftest_entry_point_reports_through_the_c_abi():
    """s2s_selftest marshals the checkpoint like s2s_create and always fills its report:
    here, with no device, the first handle cannot be made and it says so; on a GPU
    machine it runs every check (tests/test_gpu_parity.py holds the GPU assertion)."""
    import importlib
    P = pkg()
    C = importlib.import_module("swin2sr_b200.capi")
    rc, rep = C.selftest(P.weights.Weights.seeded("lightweight_sr", 0))
    assert rep.strip()
    if rc == C.S2S_OK:
        assert rep.count(" ok max-abs") == 4
    else:
        assert rc in (C.S2S_ERR_CUDA, C.S2S_ERR_UNSUPPORTED) and "create failed" in rep
