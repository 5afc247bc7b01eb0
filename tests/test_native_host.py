"""The C-ABI library: loads, exports every declared symbol, and its host-only logic (no GPU)."""
import ctypes
import os
import re

import pytest

from memintelli_flash_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    with open(os.path.join(ROOT, "include", "memintelli_b200.h")) as f:
        src = f.read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|uint64_t)\s+(mib_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    L = N.lib()
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(N.EXPORTS)
    assert b"sm_100a" in L.mib_version()


def _spec(sm, paral, qg, bfp=0):
    s = N.SliceSpec()
    s.n_slices = len(sm)
    for i, v in enumerate(sm):
        s.slice_method[i] = v
    s.bfp = bfp
    s.paral[0], s.paral[1] = paral
    s.quant_gran[0], s.quant_gran[1] = qg
    return s


def _dev(radc, rdac=4, g=4, sigma=0.0):
    d = N.DeviceSpec()
    d.hgs, d.lgs, d.g_level, d.rdac = 1e-5, 1e-8, g, rdac
    if isinstance(radc, list):
        d.n_radc = len(radc)
        for i, v in enumerate(radc):
            d.radc[i] = v
    else:
        d.n_radc, d.radc[0] = 1, radc
    d.n_read_sigma, d.read_sigma[0] = 1, sigma
    return d


def _kg(k, p=32, qg=128):
    kg = N.KGeom()
    kg.k, kg.p, kg.pp = k, p, max(32, p)
    kg.kp = -(-k // qg) * qg
    kg.kt = kg.kp // p
    return kg


def _plan(xs, ws, kg, dev):
    mode, n = N.c_i32(0), N.c_i32(0)
    rc = N.lib().mib_adc_plan(xs, ws, kg, dev, mode, n, None)
    return rc, mode.value, n.value


SM = [1, 1, 2, 2, 2]


def test_adc_plan_dyadic_uses_magic_rounding():
    rc, mode, n = _plan(_spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 32), (128, 128)), _kg(500), _dev(4096))
    assert rc == 0 and mode == 0 and n == 0


def test_adc_plan_non_dyadic_needs_table():
    xs, ws, kg, dev = _spec(SM, (1, 32), (1, 64)), _spec(SM, (32, 32), (64, 64)), _kg(100, qg=64), _dev(1024)
    rc, mode, n = _plan(xs, ws, kg, dev)
    assert rc == 0 and mode & N.MODE_LUT and n == 5 * 289
    table = (N.c_i32 * n)()
    mode_c, n_c = N.c_i32(0), N.c_i32(0)
    assert N.lib().mib_adc_plan(xs, ws, kg, dev, mode_c, n_c, table) == 0
    # round_half_even(S * 1023 / 288) for every reachable S of one slice
    assert list(table)[:289] == [round(s * 1023 / 288) for s in range(289)]


def test_split_k_workspace_choice():
    xs, ws, kg, dev = _spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 32), (128, 128)), _kg(500), _dev(4096)
    f = N.c_i64(-1)
    assert N.lib().mib_mvm_workspace(400, 600, xs, ws, kg, dev, f) == 0
    assert f.value > 0 and f.value % (400 * 600) == 0            # 52 output tiles: split the 16 K tiles
    assert N.lib().mib_mvm_workspace(16384, 3072, xs, ws, _kg(1024), dev, f) == 0
    # 8192 output tiles: no split-K; their last wave of 52 tiles is cut into 2 K ranges
    assert f.value == 52 * 2 * 128 * 48


def test_split_k_balances_a_partly_idle_last_wave():
    """352 output tiles (2048 x 1024 at 48 columns) fill 2.38 waves of 148 SMs: split in two they run as
    5 half-length waves instead of 3 full ones, so the plan asks for two partial outputs."""
    xs, ws, dev = _spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 32), (128, 128)), _dev(4096)
    f = N.c_i64(-1)
    assert N.lib().mib_mvm_workspace(2048, 1024, xs, ws, _kg(2048), dev, f) == 0
    assert f.value == 2 * 2048 * 1024
    assert N.lib().mib_mvm_workspace(4096, 1024, xs, ws, _kg(2048), dev, f) == 0
    assert f.value == 0                                           # 704 tiles: 4.76 waves, a split saves < 10%


def test_tail_split_spreads_a_nearly_empty_last_wave():
    """2816 output tiles (16384 x 1024 at 48 columns) take 20 waves of 148 SMs, the last holding 4 tiles:
    the persistent launch steps 19 waves of whole tiles and cuts the 4 remaining ones into 16 ranges of
    4 K tiles (one rescale group each), 64 partial tiles of 128 x 48 for the tail reduction.  A last wave
    at least half full is not cut."""
    xs, ws, dev = _spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 32), (128, 128)), _dev(4096)
    f = N.c_i64(-1)
    assert N.lib().mib_mvm_workspace(16384, 1024, xs, ws, _kg(2048), dev, f) == 0
    assert f.value == 4 * 16 * 128 * 48
    assert N.lib().mib_mvm_workspace(16384, 6144, xs, ws, _kg(1024), dev, f) == 0
    assert f.value == 0                                           # 16384 tiles: last wave 104 of 148


def test_adc_plan_noisy_skips_table():
    rc, mode, n = _plan(_spec(SM, (1, 32), (1, 64)), _spec(SM, (32, 32), (64, 64)), _kg(100, qg=64),
                        _dev(1024, sigma=0.05))
    assert rc == 0 and n == 0


def test_adc_plan_radc_list_length_checked():
    rc, _, _ = _plan(_spec([1, 1, 2, 2], (32, 32), (64, 64)), _spec([1, 1, 2, 2], (32, 32), (64, 64)),
                     _kg(100, qg=64), _dev([4096, 2048, 1024]))
    assert rc == N.MIB_ERR_PARAM
    assert b"must match number of weight slices" in N.lib().mib_last_error()


def test_slice_method_first_bit_checked():
    rc, _, _ = _plan(_spec([2, 2, 2], (1, 32), (1, 64)), _spec(SM, (32, 32), (64, 64)), _kg(100, qg=64), _dev(4096))
    assert rc == N.MIB_ERR_PARAM
    assert b"first bit" in N.lib().mib_last_error()
    with pytest.raises(ValueError):
        N.check(rc)


def test_mvm_rejects_bad_arguments_before_any_device_work():
    xs, ws = _spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 64), (128, 128))
    rc = N.lib().mib_mvm(None, None, 10, xs, None, None, 10, ws, _kg(128), _dev(4096), 0, None, 0, None, None,
                         None, None, None, 0, None)
    assert rc == N.MIB_ERR_PARAM


def test_fused_producers_and_attention_prep_check_arguments_on_the_host():
    L = N.lib()
    fake = ctypes.c_void_p(0x1000)          # never dereferenced: every call below fails its host checks
    xs = _spec(SM, (1, 32), (1, 128))
    assert L.mib_slice_rmsnorm_input(None, 1, 4, 128, 512, 128, fake, 1e-6, xs, _kg(128), 4, 0, fake, fake, fake,
                                     None, None, None) == N.MIB_ERR_PARAM
    assert L.mib_slice_rmsnorm_input(fake, 1, 4, 128, 512, 128, None, 1e-6, xs, _kg(128), 4, 0, fake, fake, fake,
                                     None, None, None) == N.MIB_ERR_PARAM
    assert L.mib_slice_swiglu_input(fake, 1, 4, 128, 1024, 256, 64, xs, _kg(128), 4, 0, fake, fake, fake, None,
                                    None, None) == N.MIB_ERR_SHAPE
    assert b"overlap" in L.mib_last_error()
    args = (fake, 8, 4096, 8, 16, 8, 128, fake, fake, 1e-6, fake, fake, fake, fake, fake, None)
    assert L.mib_qk_norm_rope_bf16(*args[:6], 96, *args[7:]) == N.MIB_ERR_UNSUPPORTED
    assert L.mib_qk_norm_rope_bf16(fake, 8, 4000, *args[3:]) == N.MIB_ERR_SHAPE
    assert L.mib_qk_norm_rope_bf16(None, *args[1:]) == N.MIB_ERR_PARAM


def test_engine_parameters_checked_by_every_plan_entry():
    """rdac or g_level below 2 make the ADC divisor zero: every entry point that plans an MVM returns
    MIB_ERR_PARAM with the reference's message instead of dividing by it."""
    L = N.lib()
    xs, ws, kg = _spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 32), (128, 128)), _kg(256)
    fake = ctypes.c_void_p(0x1000)          # never dereferenced: the calls fail their host checks
    for bad, msg in ((_dev(4096, rdac=1), b"DAC"), (_dev(4096, g=1), b"conductance levels")):
        rc, _, _ = _plan(xs, ws, kg, bad)
        assert rc == N.MIB_ERR_PARAM and msg in L.mib_last_error()
        f = N.c_i64(-1)
        assert L.mib_mvm_workspace(64, 64, xs, ws, kg, bad, f) == N.MIB_ERR_PARAM
        assert msg in L.mib_last_error()
        lay = N.OutLayout(64, 0, 64, 1)
        assert L.mib_mvm_static_scratch(fake, fake, 64, xs, fake, fake, 64, ws, kg, bad, 0, None, 0, fake, lay,
                                        None, None) == N.MIB_ERR_PARAM
        assert msg in L.mib_last_error()
    bad_kg = _kg(256)
    bad_kg.p = 0
    rc, _, _ = _plan(xs, ws, bad_kg, _dev(4096))
    assert rc == N.MIB_ERR_PARAM


def test_static_scratch_rejects_oversized_split_before_any_launch():
    """128 x 4800 outputs fill 100 of 148 SMs: the underfilled-grid split asks for two partial outputs,
    1.23 M floats, more than the 2^20 the built-in scratch holds."""
    L = N.lib()
    xs, ws, kg, dev = _spec(SM, (1, 32), (1, 128)), _spec(SM, (32, 32), (128, 128)), _kg(1024), _dev(4096)
    f = N.c_i64(-1)
    assert L.mib_mvm_workspace(128, 4800, xs, ws, kg, dev, f) == 0
    assert f.value == 2 * 128 * 4800 > (1 << 20)
    fake = ctypes.c_void_p(0x1000)
    lay = N.OutLayout(128, 0, 4800, 1)
    assert L.mib_mvm_static_scratch(fake, fake, 128, xs, fake, fake, 4800, ws, kg, dev, 0, None, 0, fake, lay,
                                    None, None) == N.MIB_ERR_UNSUPPORTED
    assert b"built-in scratch" in L.mib_last_error()


def test_noisy_conv_slicing_and_failure_injection_check_arguments():
    L = N.lib()
    fake = ctypes.c_void_p(0x1000)
    xs = _spec(SM, (1, 32), (1, 64))
    kg = _kg(144, qg=64)                     # 16 channels x 3 x 3 = 144 columns, padded to 192
    args = (fake, 2, 16, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, xs, kg, 4, fake, fake, fake, None, None)
    assert L.mib_slice_conv_input_noisy(*args, 0.0, 1, 0, None) == N.MIB_ERR_PARAM   # no noise: use the plain entry
    assert L.mib_slice_conv_input_noisy(*args, -0.1, 1, 0, None) == N.MIB_ERR_PARAM
    assert L.mib_slice_conv_input_noisy(None, *args[1:], 0.05, 1, 0, None) == N.MIB_ERR_PARAM
    assert L.mib_test_inject_wait_expiry(0) == N.MIB_ERR_PARAM
    assert L.mib_test_inject_wait_expiry(5_000_000_000) == N.MIB_ERR_PARAM


def test_row_logsumexp_checks_arguments():
    L = N.lib()
    fake = ctypes.c_void_p(0x1000)
    assert L.mib_row_logsumexp(None, 4, 8, 8, None, 0, fake, fake, None, None) == N.MIB_ERR_PARAM
    assert L.mib_row_logsumexp(fake, 4, 8, 8, None, 0, fake, fake, fake, None) == N.MIB_ERR_PARAM   # targets needed
    assert L.mib_row_logsumexp(fake, 4, 8, 6, None, 0, fake, fake, None, None) == N.MIB_ERR_SHAPE   # ld < cols
    assert L.mib_row_logsumexp(fake, 0, 8, 8, None, 0, fake, fake, None, None) == N.MIB_ERR_SHAPE
