"""The C-ABI library on CPU: it loads, exports what the header declares, plans,
and rejects bad arguments before touching a device (no kernel is launched by
any test here: every call below fails validation first)."""
import os
import re

import pytest

from hp_rms_norm_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    syms = set()
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            syms |= set(re.findall(r"HPRN_API\s+[\w\s\*]*?\b(hprn_\w+)\s*\(", text))
    return syms


def test_header_declares_expected_symbols():
    assert header_symbols() == set(capi.EXPORTED)


def test_library_exports_every_header_symbol():
    lib = capi.load()
    for sym in header_symbols():
        assert hasattr(lib, sym), sym


def test_version_and_status_strings():
    assert capi.version() == 10000
    lib = capi.load()
    assert lib.hprn_status_string(0) == b"HPRN_OK"
    assert lib.hprn_status_string(-1) == b"HPRN_ERR_INVALID_ARGUMENT"
    assert lib.hprn_status_string(-4) == b"HPRN_ERR_CUDA"
    assert lib.hprn_status_string(99) == b"HPRN_ERR_UNKNOWN"


@pytest.mark.parametrize("rows,hidden,kind", [
    (4096, 1024, "warp"), (4096, 2048, "cta"), (4096, 4096, "cta"), (4096, 8192, "cta"),
    (4096, 16384, "cta"), (4096, 32768, "cta"), (1, 8192, "cta"), (4, 65536, "cluster"),
    (4, 1 << 18, "twopass"), (4, 40960, "cluster"), (3, 1 << 22, "twopass"),
])
def test_plan_kinds(rows, hidden, kind):
    p = capi.plan(rows, hidden)
    assert p.startswith(kind + ":"), p
    assert ":vec32:" in p


def test_plan_is_for_the_fused_form_whatever_the_pointers():
    """hprn_rms_norm_plan plans the in-place fused op; a null residual pointer
    (planning without tensors) must not switch it to the plain form's plans."""
    assert capi.plan(4096, 16384) == capi.plan(4096, 16384, input_ptr=1 << 20,
                                               residual_ptr=1 << 21)
    assert capi.plan(4096, 16384) == "cta:vec32:vpt1:tpr1024:cluster1:rpc1"
    assert capi.plan(4096, 1024) == "warp:vec32:vpt2:tpr32:cluster1:rpc4"
    assert capi.plan(4096, 1536) == "warp:vec32:vpt3:tpr32:cluster1:rpc4"


@pytest.mark.parametrize("rows,hidden,plan", [
    (1, 1024, "cta:vec16:vpt1:tpr128:cluster1:rpc1"),
    (512, 1024, "cta:vec16:vpt1:tpr128:cluster1:rpc1"),
    (33, 1536, "cta:vec16:vpt1:tpr192:cluster1:rpc1"),
    (128, 2048, "cta:vec16:vpt1:tpr256:cluster1:rpc1"),
    (513, 1024, "warp:vec32:vpt2:tpr32:cluster1:rpc4"),
    (512, 512, "warp:vec32:vpt1:tpr32:cluster1:rpc4"),
    (512, 4096, "cta:vec32:vpt1:tpr256:cluster1:rpc1"),
])
def test_small_batch_plans(rows, hidden, plan):
    """Decode-sized batches of fused rows of 528-2048 elements take one CTA per
    row at 16-byte vectors; larger batches, shorter rows and longer rows keep
    their own rules."""
    assert capi.plan(rows, hidden) == plan


@pytest.mark.parametrize("hidden,plan", [
    # rows past one CTA: eight-CTA clusters, one vector per thread up to 512
    # vectors per CTA, else two (the long-row sweep's fit)
    (40960, "cluster:vec32:vpt1:tpr320:cluster8:rpc1"),
    (65536, "cluster:vec32:vpt1:tpr512:cluster8:rpc1"),
    (98304, "twopass:vec32:vpt4:tpr512:cluster1:rpc1"),
    (131072, "twopass:vec32:vpt4:tpr128:cluster8:rpc1"),
    (262144, "twopass:vec32:vpt4:tpr128:cluster8:rpc1"),
    (262160, "twopass:vec32:vpt4:tpr256:cluster8:rpc1"),
    # short rows: several rows per warp, one vector per lane
    (16, "warp:vec32:vpt1:tpr1:cluster1:rpc256"),
    (64, "warp:vec32:vpt1:tpr4:cluster1:rpc64"),
    (256, "warp:vec32:vpt1:tpr16:cluster1:rpc16"),
    (512, "warp:vec32:vpt1:tpr32:cluster1:rpc4"),
    # the config-1 sweep's regimes
    (20480, "cta:vec32:vpt4:tpr320:cluster1:rpc1"),
    (24576, "cta:vec32:vpt2:tpr768:cluster1:rpc1"),
    (32768, "cta:vec32:vpt2:tpr1024:cluster1:rpc1"),
])
def test_fitted_plans(hidden, plan):
    assert capi.plan(4096, hidden) == plan


def test_tuner_tma_candidates_fit_a_cta():
    from hp_rms_norm_b200 import tune

    for hidden, residual in ((1024, True), (4096, True), (16384, True), (16384, False)):
        cands = tune.tma_candidates(hidden, residual)
        assert cands, hidden
        for c in cands:
            f = dict(re.findall(r"([a-z]+)(\d+)", c))
            vec, vpt, tpr, stages = (int(f[k]) for k in ("vec", "vpt", "tpr", "rpc"))
            assert tpr * vpt * (vec // 2) >= hidden, c
            assert stages * (2 if residual else 1) * hidden * 2 <= tune.TMA_SMEM, c
            load = vpt * vec // 16
            assert tpr <= (1024 if load <= 2 else 512 if load <= 4 else 256), c
    # A fused row of 32768 is a 128 KB stage: one ring slot, 32-byte vectors only.
    assert tune.tma_candidates(32768, True) == ["tma:vec32:vpt8:tpr256:cluster1:rpc1"]
    assert tune.tma_candidates(65536, True) == []  # no CTA covers it


def test_plan_vector_width_follows_alignment_and_hidden():
    assert ":vec32:" in capi.plan(8, 4096, input_ptr=256, residual_ptr=1 << 20)
    assert ":vec16:" in capi.plan(8, 4096, input_ptr=256 + 16, residual_ptr=1 << 20)
    assert ":vec8:" in capi.plan(8, 4100)
    assert ":vec4:" in capi.plan(8, 4098)
    assert ":vec2:" in capi.plan(8, 4097)
    assert ":vec16:" in capi.plan(8, 4096, input_row_stride=4104)


def test_plan_covers_every_row_length():
    """Every plan's threads x vectors x CTAs covers the row (no element dropped)."""
    for hidden in list(range(1, 300)) + [1000, 4095, 5120, 13312, 20480, 65536, 262144, 1 << 20]:
        p = capi.plan(4, hidden)
        f = dict(re.findall(r"([a-z]+)(\d+)", p))
        vec, vpt, tpr, cl = (int(f[k]) for k in ("vec", "vpt", "tpr", "cluster"))
        nvec = hidden // (vec // 2)
        assert hidden % (vec // 2) == 0, (hidden, p)
        if p.startswith("warp"):
            assert vpt * tpr >= nvec, (hidden, p)
        elif not p.startswith("twopass"):
            assert tpr * vpt * cl >= nvec, (hidden, p)


def expect_error(status_fn, status, fragment):
    with pytest.raises(capi.HprnError) as e:
        status_fn()
    assert e.value.status == status
    assert fragment in str(e.value)


def test_rms_norm_argument_errors_before_any_launch():
    F = 1 << 20  # fake device addresses: every call below must be rejected by validation
    bf = capi.DTYPE_BF16
    expect_error(lambda: capi.rms_norm(F, F, F, 4, 8, 8, 8, 1e-6, 7), capi.ERR_UNSUPPORTED_DTYPE,
                 "dtype must be kFloat16 or kBFloat16")
    expect_error(lambda: capi.rms_norm(F, F, 2 * F, -1, 8, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "rows")
    expect_error(lambda: capi.rms_norm(F, F, 2 * F, 4, 0, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "hidden_dim")
    expect_error(lambda: capi.rms_norm(0, F, 2 * F, 4, 8, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "null")
    expect_error(lambda: capi.rms_norm(F + 1, F, 2 * F, 4, 8, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "aligned")
    expect_error(lambda: capi.rms_norm(F, F, 2 * F, 4, 8, 4, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "strides")
    # residual starts inside input's rows
    expect_error(lambda: capi.rms_norm(F, F, F + 8, 4, 8, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "overlap")
    expect_error(lambda: capi.rms_norm(F, F, F, 4, 8, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "overlap")
    expect_error(lambda: capi.rms_norm(F, F + 16, 2 * F, 4, 8, 8, 8, 1e-6, bf),
                 capi.ERR_INVALID_ARGUMENT, "weight must not overlap")


def test_rms_norm_zero_rows_is_a_no_op():
    capi.rms_norm(0, 0, 0, 0, 4096, 4096, 4096, 1e-6, capi.DTYPE_BF16)


def test_relu_argument_errors_before_any_launch():
    F = 1 << 20
    bf = capi.DTYPE_BF16
    expect_error(lambda: capi.relu(F, 2 * F, 4, 8, 8, 8, 5), capi.ERR_UNSUPPORTED_DTYPE, "dtype")
    expect_error(lambda: capi.relu(F, 2 * F, -1, 8, 8, 8, bf), capi.ERR_INVALID_ARGUMENT, ">= 0")
    expect_error(lambda: capi.relu(0, 2 * F, 4, 8, 8, 8, bf), capi.ERR_INVALID_ARGUMENT, "null")
    expect_error(lambda: capi.relu(F + 2, F, 4, 8, 8, 8, bf), capi.ERR_INVALID_ARGUMENT, "overlap")
    expect_error(lambda: capi.relu(F, 2 * F, 4, 8, 4, 8, bf), capi.ERR_INVALID_ARGUMENT, "strides")
    capi.relu(0, 0, 0, 8, 8, 8, bf)  # empty: no-op


def test_plan_override_parsing():
    expect_error(lambda: capi.set_plan_override("nonsense"), capi.ERR_INVALID_ARGUMENT, "unparsable")
    capi.set_plan_override("cta:vec32:vpt2:tpr128:cluster1:rpc1")
    capi.set_plan_override("tma:vec16:vpt1:tpr128:cluster1:rpc4")
    capi.set_plan_override(None)
    assert capi.plan(4096, 4096).startswith("cta:")


@pytest.mark.parametrize("bad", [
    "default:pf4:et0", "default:pf1:et3", "default:pf1", "default:pf1:et1x",
    "cta:vec32:vpt1:tpr256:cluster1:rpc1:pf1", "cta:vec32:vpt1:tpr256:cluster1:rpc1:pf-1:et0",
    "cta:vec32:vpt1:tpr256:cluster1:rpc1 ", "cta:vec32:vpt1:tpr256:cluster1:rpc1:et1:pf1",
])
def test_plan_override_rejects_malformed_knobs(bad):
    expect_error(lambda: capi.set_plan_override(bad), capi.ERR_INVALID_ARGUMENT, "unparsable")
    capi.set_plan_override(None)


def test_plan_override_knobs_are_echoed():
    """Launch knobs (L2 prefetch scope, trigger point) are implied by the plan
    unless an override names them: "default:pf<p>:et<e>" keeps the default plan
    and sets only the knobs; a full plan may carry them as a suffix."""
    base = capi.plan(4096, 4096)
    assert ":pf" not in base
    try:
        capi.set_plan_override("default:pf0:et1")
        assert capi.plan(4096, 4096) == base + ":pf0:et1"
        assert capi.plan(4096, 1024) == capi.plan(4096, 1024).split(":pf")[0] + ":pf0:et1"
        capi.set_plan_override("cta:vec32:vpt2:tpr128:cluster1:rpc1:pf1:et0")
        assert capi.plan(4096, 4096) == "cta:vec32:vpt2:tpr128:cluster1:rpc1:pf1:et0"
        capi.set_plan_override("cta:vec32:vpt2:tpr128:cluster1:rpc1")
        assert capi.plan(4096, 4096) == "cta:vec32:vpt2:tpr128:cluster1:rpc1"
    finally:
        capi.set_plan_override(None)
    assert capi.plan(4096, 4096) == base


def test_wait_timeouts_needs_a_count_pointer():
    lib = capi.load()
    assert lib.hprn_wait_timeouts(None, 0) == capi.ERR_INVALID_ARGUMENT


def test_stall_hook_arguments():
    """The bounded-wait test hook takes a row (or -1: off) and a limit of at
    most one second; it only records settings, so it runs without a GPU."""
    expect_error(lambda: capi.test_stall_bulk_copy(0, 2_000_000_000), capi.ERR_INVALID_ARGUMENT,
                 "one second")
    capi.test_stall_bulk_copy(3, 1_000_000)
    capi.test_stall_bulk_copy(None)
