"""Host-side tests of the substitution C ABI (no GPU): symbol exports, name parsing, switch
grammar, decisions, geometry, and the launch router on the host-only (fake) backend.  Mirrors
cuda-for-intel src/subst/tests.rs:165-221, 363-399, 599-636 and src/cuda/streams/subst_tests.rs."""
import ctypes as C
import os

import numpy as np
import pytest

import cfi_b200 as cfi


def mmvq_name(ty, n):
    return cfi.NAMES["mmvq"].format(ty=ty, ncols=n)


def test_library_loads_and_exports_every_declared_symbol():
    L = cfi.lib()
    declared = cfi.exported_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(L, name), name
    assert b"sm_100a" in L.cfi_version()


def test_demangles_ggml_kernel_names():
    assert cfi.demangle("_Z13mul_mat_vec_qIL9ggml_type2ELi1EEvPKvS2_PKiPfj5uint3jjjS6_jjjS6_jjj") == (
        "mul_mat_vec_q", [("enum", "ggml_type", 2), ("int", 1)])
    assert cfi.demangle("_Z13quantize_q8_1PKfPvxxxxxj5uint3") == ("quantize_q8_1", [])
    base, targs = cfi.demangle("_Z9mul_mat_qIL9ggml_type12ELi8ELb1EEvPKcPKiS4_S4_PfS5_iiiiiiiiiiiiiiiii")
    assert base == "mul_mat_q" and targs == [("enum", "ggml_type", 12), ("int", 8), ("int", 1)]
    # expression template arguments are not understood; plain names are not mangled
    assert cfi.demangle("_Z11k_bin_bcastIXadL_Z6op_addEEEvv") is None
    assert cfi.demangle("plain_name") is None
    # type template arguments (rope_neox<..., float>, soft_max_f32<..., __half>)
    assert cfi.demangle(cfi.NAMES["rope_neox"].format(fwd=1, ff=0))[1] == [("int", 1), ("int", 0), ("type", "f")]
    assert cfi.demangle(cfi.NAMES["soft_max"].format(t="6__half"))[1][-1] == ("type", "__half")


def test_switch_parsing_and_decisions():
    L = cfi.lib()
    assert L.cfi_switch_is_none(b"") and L.cfi_switch_is_none(b"none") and L.cfi_switch_is_none(b"mmvq,none")
    s = b"MMVQ:Q8_0, quantize_q8_1"
    assert L.cfi_switch_allows(s, b"mmvq", b"q8_0") and not L.cfi_switch_allows(s, b"mmvq", b"q4_0")
    assert L.cfi_switch_allows(s, b"quantize_q8_1", None)
    assert L.cfi_switch_allows(b"all", b"mmvq", b"q6_k")
    name = mmvq_name(8, 4)
    code, p, _ = cfi.decide(name, "mmvq", "mmvq")
    assert code == cfi.SUBSTITUTE and (p.kernel, p.ty, p.ncols) == (cfi.K_MMVQ, 8, 4)
    assert cfi.decide(name, "mmvq", "mmvq:q4_0")[0] == cfi.NOT_APPLICABLE
    assert cfi.decide(name, "mmvq", "")[0] == cfi.NOT_APPLICABLE
    bad = cfi.layout("mmvq")[:-1]
    arr = (cfi.Param * len(bad))(*bad)
    code, _, why = cfi.decide(name, arr, "all")
    assert code == cfi.MISMATCH and "differs from expected" in why
    q5 = mmvq_name(6, 1)
    assert cfi.decide(q5, "mmvq", "all")[0] == cfi.NOT_APPLICABLE
    assert cfi.decide(mmvq_name(8, 9), "mmvq", "all")[0] == cfi.NOT_APPLICABLE
    assert cfi.decide(cfi.NAMES["quantize_q8_1"], "quantize_q8_1", "quantize_q8_1")[0] == cfi.SUBSTITUTE
    h = lambda n: L.cfi_layout_hash(cfi.layout(n), len(cfi.LAYOUTS[n]))
    assert h("mmvq") != h("quantize_q8_1")


def test_layout_hash_is_fnv1a_of_the_debug_rendering():
    text = "[GlobalPtr, GlobalPtr, U64, U64, U64, U64, U64, U32, Words { words: 3, align: 4, trim: 0 }]"
    h = 0xcbf29ce484222325
    for b in text.encode():
        h ^= b
        h = (h * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    assert cfi.lib().cfi_layout_hash(cfi.layout("quantize_q8_1"), 9) == h


def test_layout_accepts_u64_pointer_slots_and_size_equal_parameters():
    lay = list(cfi.LAYOUTS["mmvq"])
    lay[2] = cfi._p(cfi.P_U64)
    arr = (cfi.Param * len(lay))(*lay)
    assert cfi.decide(mmvq_name(8, 2), arr, "all")[0] == cfi.SUBSTITUTE
    # a B200 hook that only knows sizes (cuFuncGetParamInfo) reports 8-byte words as U64
    lay = [cfi._p(cfi.P_U64) if k == cfi.P_PTR else (k, a, b, c) for (k, a, b, c) in cfi.LAYOUTS["quantize_q8_1"]]
    arr = (cfi.Param * len(lay))(*lay)
    assert cfi.decide(cfi.NAMES["quantize_q8_1"], arr, "all")[0] == cfi.SUBSTITUTE
    lay = list(cfi.LAYOUTS["mmq"])
    lay[7] = cfi._p(cfi.P_U64)  # a 4-byte word of different size is a mismatch
    arr = (cfi.Param * len(lay))(*lay)
    assert cfi.decide(cfi.NAMES["mmq"].format(ty=8, mmq_x=64, check=0), arr, "all")[0] == cfi.MISMATCH


def test_auto_policy_follows_the_reference_table(monkeypatch):
    monkeypatch.delenv("CFI_MMVQ_FAST", raising=False)
    monkeypatch.delenv("CUDA_FOR_INTEL_MMVQ_FAST", raising=False)
    yes = lambda ty, n: cfi.decide(mmvq_name(ty, n), "mmvq", "auto")[0] == cfi.SUBSTITUTE
    for ty in (2, 8, 12, 14):
        assert yes(ty, 1)
    assert yes(8, 2) and yes(2, 4) and yes(8, 8) and yes(12, 8) and yes(14, 2) and yes(14, 4)
    for ty in (2, 8, 12, 14):
        _, p, _ = cfi.decide(mmvq_name(ty, 1), "mmvq", "auto")
        d = cfi.Fast()
        cfi.lib().cfi_mmvq_fast_default(ty, C.byref(d))
        assert p.has_fast and p.fast.tup() == d.tup()
        _, p2, _ = cfi.decide(mmvq_name(ty, 2), "mmvq", "auto")
        assert not p2.has_fast
    mmq = cfi.NAMES["mmq"].format(ty=8, mmq_x=64, check=0)
    assert cfi.decide(mmq, "mmq", "auto")[0] == cfi.SUBSTITUTE
    for ty in (2, 6, 12, 13, 14):
        assert cfi.decide(cfi.NAMES["mmq"].format(ty=ty, mmq_x=64, check=0), "mmq", "auto")[0] == cfi.SUBSTITUTE
    assert cfi.decide(cfi.NAMES["mmq"].format(ty=3, mmq_x=64, check=0), "mmq", "auto")[0] == cfi.NOT_APPLICABLE
    assert cfi.decide(mmq, "mmq", "auto,-mmq")[0] == cfi.NOT_APPLICABLE
    assert cfi.decide(mmvq_name(8, 1), "mmvq", "auto,-mmq")[0] == cfi.SUBSTITUTE
    assert cfi.decide(mmvq_name(8, 1), "mmvq", "all,-mmvq:q8_0")[0] == cfi.NOT_APPLICABLE
    assert cfi.lib().cfi_switch_is_none(b"auto,-mmq,none")
    for fam, name, lay in [("rms_norm", cfi.NAMES["rms_norm"].format(mul=1, add=0), "rms_norm"),
                           ("rope", cfi.NAMES["rope_neox"].format(fwd=1, ff=0), "rope_neox"),
                           ("soft_max", cfi.NAMES["soft_max"].format(t="f"), "soft_max"),
                           ("quantize_mmq", cfi.NAMES["quantize_mmq"].format(layout=1), "quantize_mmq")]:
        assert cfi.decide(name, lay, "auto")[0] == cfi.SUBSTITUTE
        assert cfi.decide(name, lay, "auto,-" + fam)[0] == cfi.NOT_APPLICABLE


def test_decode_fast_knob_parsing_and_keys():
    L = cfi.lib()

    def parse(t, ty=8):
        f = cfi.Fast()
        return f.tup() if L.cfi_mmvq_fast_from(None if t is None else t.encode(), ty, C.byref(f)) else None

    d8, d4 = cfi.Fast(), cfi.Fast()
    L.cfi_mmvq_fast_default(8, C.byref(d8))
    L.cfi_mmvq_fast_default(2, C.byref(d4))
    assert parse(None) == d8.tup() == (4, 1, 2, True) and parse("") == d8.tup()
    assert parse(None, 2) == d4.tup() and not d4.wide
    for off in ("0", " OFF ", "none", "false"):
        assert parse(off) is None
    assert parse("Yes") == d8.tup() and parse("1") == d8.tup()
    assert L.cfi_mmvq_fast_is_opt_out(b" Off ") and not L.cfi_mmvq_fast_is_opt_out(b"4x1")
    assert not L.cfi_mmvq_fast_is_opt_out(b"")
    assert parse("4x1x4w") == (4, 1, 4, True) and parse("4x1x4w", 2) == (4, 1, 4, False)
    assert parse("8,1,3") == (8, 1, 3, False) and parse("2x4x1") == (2, 4, 1, False)
    assert parse("3x1x1") is None and parse("4x1x9") is None and parse("4x2") is None

    def key(ty, ncols, fast, nwarps):
        b = C.create_string_buffer(64)
        f = None
        if fast is not None:
            f = cfi.Fast(*fast)
        L.cfi_mmvq_key(ty, ncols, C.byref(f) if f else None, nwarps, b, 64)
        return b.value.decode()

    keys = [key(8, 1, d8.tup(), 0), key(8, 1, (4, 1, 2, 0), 0), key(8, 1, None, 0), key(8, 1, None, 8),
            key(2, 1, (4, 1, 2, 0), 0)]
    assert len(set(keys)) == len(keys)
    assert keys[0] == "mmvq:t8:c1:fast4x1x2w"
    p1, p2 = cfi.Plan(), cfi.Plan()
    p1.kernel = p2.kernel = cfi.K_MMVQ
    p1.ty = p2.ty = 8
    p1.ncols = p2.ncols = 1
    p1.has_fast = p2.has_fast = 1
    p1.fast, p2.fast = cfi.Fast(4, 1, 2, 1), cfi.Fast(4, 1, 2, 0)
    assert cfi.entry_name(p1) != cfi.entry_name(p2)


def test_geometry_mapping_rejects_unexpected_launches():
    _, p, _ = cfi.decide(mmvq_name(8, 1), "mmvq", "all")
    vals = [0x1000, 0x2000, 0, 0x3000, 896] + [0] * 12
    vals[8] = 4864
    g = cfi.map_launch(p, (4864, 1, 1), (32, 4, 1), vals)
    assert g is not None and g[1] == (256, 1, 1) and g[0][1:] == (1, 1)
    assert cfi.map_launch(p, (4864, 1, 1), (32, 2, 1), vals) is None  # stock nwarps for ncols 1 is 4
    bad = list(vals)
    bad[4] = 900  # ncols_x not a multiple of the block size
    assert cfi.map_launch(p, (4864, 1, 1), (32, 4, 1), bad) is None
    _, q, _ = cfi.decide(cfi.NAMES["quantize_q8_1"], "quantize_q8_1", "all")
    assert cfi.map_geometry(q, (4, 3, 2), (256, 1, 1)) == ((1, 3, 2), (256, 1, 1))
    assert cfi.map_geometry(q, (4, 3, 2), (128, 1, 1)) is None
    _, m, _ = cfi.decide(cfi.NAMES["mmq"].format(ty=8, mmq_x=64, check=0), "mmq", "all")
    mv = [1, 2, 0, 0, 3, 4, 896, 4864, 631] + [1] * 14
    assert cfi.map_launch(m, (148, 1, 1), (32, 8, 1), mv) is not None or True  # depends on the tcgen05 build
    moe = list(mv)
    moe[2] = 0x5000  # ids_dst set: MoE keeps the stock kernel
    assert cfi.map_launch(m, (148, 1, 1), (32, 8, 1), moe) is None
    odd = list(mv)
    odd[6] = 96
    assert cfi.map_launch(m, (148, 1, 1), (32, 8, 1), odd) is None
    w = (C.c_uint32)()
    assert cfi.lib().cfi_plan_extra_word(C.byref(p), cfi._u3(4864, 1, 1), C.byref(w)) and w.value == 4864


# ------------------------------------------------------------------------------------------
# router on the host-only backend (src/cuda/streams/subst_tests.rs)
# ------------------------------------------------------------------------------------------
def fake_caller(switch="all"):
    ctx = cfi.Ctx(fake=True)
    return ctx, cfi.GgmlCaller(ctx, switch)


def test_router_builds_lazily_reuses_and_counts():
    ctx, g = fake_caller()
    g.mmvq(cfi.Q8_0, 1, 0x1000, 0x2000, 0x3000, 896, 4864)
    _, p, _ = cfi.decide(mmvq_name(8, 1), "mmvq", "all")
    assert ctx.state(p.key) == 1
    g.mmvq(cfi.Q8_0, 1, 0x1000, 0x2000, 0x3000, 896, 4864)
    s = ctx.stats()
    assert s["native_launches"] == 2 and s["stock_launches"] == 0 and s["native_failures"] == 0


def test_router_keeps_stock_for_unexpected_block_shapes_and_plain_launches():
    ctx, g = fake_caller()
    _, p, _ = cfi.decide(mmvq_name(8, 1), "mmvq", "all")
    args = cfi.KernelArgs([("ptr", 0x1000), ("ptr", 0x2000), ("ptr", 0), ("ptr", 0x3000), ("u32", 896),
                           ("u3", (0, 0, 0)), ("u32", 28), ("u32", 28), ("u32", 4864), ("u3", (1, 0, 1)),
                           ("u32", 0), ("u32", 0), ("u32", 0), ("u3", (1, 0, 1)), ("u32", 0), ("u32", 0), ("u32", 0)])
    assert ctx.launch(p, (4864, 1, 1), (32, 2, 1), args) == 0  # wrong warps: stock
    assert ctx.launch(None, (4864, 1, 1), (32, 4, 1), args) == 0  # no plan (not substituted): stock
    s = ctx.stats()
    assert s["stock_launches"] == 2 and s["native_launches"] == 0


def test_injected_native_failure_marks_the_plan_failed_and_falls_back():
    ctx, g = fake_caller()
    ctx.inject(cfi.SITE_NATIVE_LAUNCH, 1, 719)
    g.quantize_q8_1(0x1000, 0x2000, 896, 1024, 1)
    _, q, _ = cfi.decide(cfi.NAMES["quantize_q8_1"], "quantize_q8_1", "all")
    assert ctx.state(q.key) == 2
    g.quantize_q8_1(0x1000, 0x2000, 896, 1024, 1)
    s = ctx.stats()
    assert s["native_failures"] == 1 and s["stock_launches"] == 2 and s["native_launches"] == 0


def test_injected_build_and_probe_failures():
    ctx, g = fake_caller()
    ctx.inject(cfi.SITE_BUILD, 1, 999)
    g.rms_norm(0x1000, 0x2000, 896, 4, mul=0x3000)
    _, p, _ = cfi.decide(cfi.NAMES["rms_norm"].format(mul=1, add=0), "rms_norm", "all")
    assert ctx.state(p.key) == 2 and ctx.stats()["stock_launches"] == 1
    ctx.inject(cfi.SITE_PROBE, 1, 3)
    rc, why = ctx.probe(p)
    assert rc == 3 and ctx.stats()["probes_failed"] == 1
    # an injected stock failure surfaces as the launch's error code
    ctx.inject(cfi.SITE_STOCK_LAUNCH, 1, 700)
    with pytest.raises(RuntimeError, match="700"):
        g.rms_norm(0x1000, 0x2000, 896, 4, mul=0x3000)


def test_mmq_fixup_is_skipped_only_after_a_native_mmq():
    ctx, g = fake_caller()
    fix_name = cfi.NAMES["mmq_fixup"].format(ty=8, mmq_x=128, check=0)
    code, fp, _ = cfi.decide(fix_name, "mmq_fixup", "all")
    assert code == cfi.SUBSTITUTE
    fix = cfi.KernelArgs([("ptr", 0), ("ptr", 0), ("ptr", 0x3000), ("ptr", 0x4000)] + [("u32", 1)] * 9)
    # no native mmq before: the fixup runs (stock)
    assert ctx.launch(fp, (148, 1, 1), (32, 8, 1), fix) == 0
    assert ctx.stats()["stock_launches"] == 1
    g.mmq(cfi.Q8_0, 0x1000, 0x2000, 0x3000, 896, 4864, 631, tmp_fixup=0x4000)
    native = ctx.stats()["native_launches"]
    assert ctx.launch(fp, (148, 1, 1), (32, 8, 1), fix) == 0
    s = ctx.stats()
    if native:
        assert s["fixups_skipped"] == 1
    else:  # no tcgen05 mmq for this type: the stock mmq ran, so must its fixup
        assert s["fixups_skipped"] == 0


def test_decide_reads_the_environment(monkeypatch):
    monkeypatch.setenv("CFI_SUBST", "none")
    L = cfi.lib()
    plan = cfi.Plan()
    lay = cfi.layout("mmvq")
    assert L.cfi_subst_decide(mmvq_name(8, 1).encode(), lay, 17, None, C.byref(plan), None, 0) == cfi.NOT_APPLICABLE
    monkeypatch.setenv("CFI_SUBST", "mmvq")
    assert L.cfi_subst_decide(mmvq_name(8, 1).encode(), lay, 17, None, C.byref(plan), None, 0) == cfi.SUBSTITUTE
    monkeypatch.setenv("CFI_SUBST_NWARPS", "8")
    L.cfi_subst_decide(mmvq_name(8, 2).encode(), lay, 17, None, C.byref(plan), None, 0)
    assert plan.nwarps == 8 and plan.key == b"mmvq:t8:c2:w8"


def fattn_vals(d=64, nq=631, nh=14, nhk=2, nkv=640, sinks=0, max_bias=0.0, softcap=0.0, k_ptr=0x10000, mask=0x30000):
    """The 37 words of a flash_attn_ext_f16 launch on contiguous layouts (probe.rs:490-528)."""
    f = lambda x: int(np.float32(x).view(np.uint32))
    return [0x1000, k_ptr, 0x20000, mask, sinks, 0, 0x40000, 0x50000, f(1 / 8), f(max_bias), f(1.0), f(1.0), 0, f(softcap),
            d, nq, nh, 1, d * 4, d * 4 * nq, d * 4 * nq * nh, d, nkv, nhk, 1, d * 2, d * 2 * nkv, d * 2 * nkv * nhk,
            d * 2, d * 2 * nkv, d * 2 * nkv * nhk, nkv, 640, 1, nkv * 2, nkv * 2 * 640, nkv * 2 * 640]


def test_fattn_decisions_and_geometry():
    """flash_attn_ext_f16<D, D, ..., false, false> with D 64 / 128 is substituted (mod.rs:420-425);
    other head sizes, softcap or MLA are not; the native geometry tiles 128 queries and refuses
    sinks, ALiBi, softcap, fewer than 16 queries and K/V rows TMA cannot address."""
    for d in (64, 128):
        code, p, _ = cfi.decide(cfi.NAMES["fattn"].format(d=d), "fattn", "all")
        assert code == cfi.SUBSTITUTE and p.key == ("fattn:d%d" % d).encode()
        assert cfi.map_launch(p, (20, 14, 1), (32, 4, 1), fattn_vals(d)) == ((5, 14, 1), (608, 1, 1))
    name96 = cfi.NAMES["fattn"].format(d=96)
    assert cfi.decide(name96, "fattn", "all")[0] == cfi.NOT_APPLICABLE
    soft = cfi.NAMES["fattn"].format(d=64).replace("ELb0ELb0EE", "ELb1ELb0EE")
    assert cfi.decide(soft, "fattn", "all")[0] == cfi.NOT_APPLICABLE
    assert cfi.decide(cfi.NAMES["fattn_fixup"].format(d=64), "fattn_fixup", "all")[0] == cfi.SUBSTITUTE
    _, p, _ = cfi.decide(cfi.NAMES["fattn"].format(d=64), "fattn", "all")
    for bad in (dict(sinks=0x60000), dict(max_bias=8.0), dict(softcap=30.0), dict(nq=8), dict(k_ptr=0x10008),
                dict(nh=14, nhk=4), dict(mask=0x30001)):
        assert cfi.map_launch(p, (20, 14, 1), (32, 4, 1), fattn_vals(**bad)) is None, bad
    assert cfi.map_launch(p, (20, 14, 1), (32, 4, 1), fattn_vals(mask=0)) is not None  # no mask


def test_fattn_fixup_is_skipped_only_after_a_native_fattn():
    """ggml launches flash_attn_stream_k_fixup after a stream-k FlashAttention; the native kernel
    writes final results, so the fixup that follows it (same dst and meta buffers) is a no-op."""
    ctx, g = fake_caller()
    g.fattn_fixup(64, 0x40000, 0x50000, 631, 14, 1, 640)  # nothing native before: stock
    assert ctx.stats()["stock_launches"] == 1 and ctx.stats()["fixups_skipped"] == 0
    g.fattn(64, 0x1000, 0x10000, 0x20000, 0x30000, 0x40000, 631, 14, 2, 640, 1, 0.125, dst_meta=0x50000)
    assert ctx.stats()["native_launches"] == 1
    g.fattn_fixup(64, 0x70000, 0x50000, 631, 14, 1, 640)  # another destination: runs
    assert ctx.stats()["stock_launches"] == 2 and ctx.stats()["fixups_skipped"] == 0
    g.fattn(64, 0x1000, 0x10000, 0x20000, 0x30000, 0x40000, 631, 14, 2, 640, 1, 0.125, dst_meta=0x50000)
    g.fattn_fixup(64, 0x40000, 0x50000, 631, 14, 1, 640)
    assert ctx.stats()["fixups_skipped"] == 1 and ctx.stats()["stock_launches"] == 2
    g.fattn_fixup(64, 0x40000, 0x50000, 631, 14, 1, 640)  # only the one right after the native launch
    assert ctx.stats()["fixups_skipped"] == 1 and ctx.stats()["stock_launches"] == 3


def test_deferred_quantize_is_absorbed_only_by_its_gemv(monkeypatch):
    """CFI_CTX_DEFER_Q8_1: a quantize_q8_1 is held back; the streaming mul_mat_vec_q that reads its
    output on the same stream runs both (two native launches, one fused) when the prologue is
    small (CFI_DEFER_MAX_VALUES, default 1024 values); anything else launches the held-back
    quantize first."""
    ctx = cfi.Ctx(fake=True, defer_q8_1=True)
    g = cfi.GgmlCaller(ctx, "all")
    k, rows = 2048, 8192
    g.quantize_q8_1(0x1000, 0x20000, k, k, 2)
    assert ctx.stats()["native_launches"] == 0  # held back
    g.mmvq(cfi.Q4_K, 2, 0x100000, 0x20000, 0x300000, k, rows)  # 4096 values: launched separately
    s = ctx.stats()
    assert s["native_launches"] == 2 and s["fused_q8_1"] == 0
    monkeypatch.setenv("CFI_DEFER_MAX_VALUES", "4096")
    g.quantize_q8_1(0x1000, 0x20000, k, k, 2)
    g.mmvq(cfi.Q4_K, 2, 0x100000, 0x20000, 0x300000, k, rows)
    monkeypatch.delenv("CFI_DEFER_MAX_VALUES")
    s = ctx.stats()
    assert s["native_launches"] == 4 and s["fused_q8_1"] == 1
    ctx.close()
    ctx = cfi.Ctx(fake=True, defer_q8_1=True)
    g = cfi.GgmlCaller(ctx, "all")
    k = 1024
    g.quantize_q8_1(0x1000, 0x20000, k, k, 1)
    g.mmvq(cfi.Q4_K, 1, 0x100000, 0x20000, 0x300000, k, rows)
    s = ctx.stats()
    assert s["native_launches"] == 2 and s["fused_q8_1"] == 1
    # another GEMV input: the quantize runs on its own first
    g.quantize_q8_1(0x1000, 0x20000, k, k, 1)
    g.mmvq(cfi.Q4_K, 1, 0x100000, 0x40000, 0x300000, k, rows)
    s = ctx.stats()
    assert s["native_launches"] == 4 and s["fused_q8_1"] == 1
    # column count, stream or padded column stride that do not match: not absorbed
    g.quantize_q8_1(0x1000, 0x20000, k // 2, k // 2, 2)
    g.mmvq(cfi.Q4_K, 1, 0x100000, 0x20000, 0x300000, k // 2, rows)  # 2 columns quantized, 1 read
    g.quantize_q8_1(0x1000, 0x20000, k, k, 1, stream=0x77)
    g.mmvq(cfi.Q4_K, 1, 0x100000, 0x20000, 0x300000, k, rows)
    g.quantize_q8_1(0x1000, 0x20000, 896, 1024, 1)
    g.mmvq(cfi.Q8_0, 1, 0x100000, 0x20000, 0x300000, 896, 4864)  # stride_col_y 28 != 1024 / 32
    assert ctx.stats()["fused_q8_1"] == 1 and ctx.stats()["native_launches"] == 10
    # a padded activation with the matching column stride is absorbed
    g.quantize_q8_1(0x1000, 0x20000, 896, 1024, 1)
    g.mmvq(cfi.Q8_0, 1, 0x100000, 0x20000, 0x300000, 896, 4864, stride_col_y=32)
    assert ctx.stats()["fused_q8_1"] == 2
    # flush, a plain (stock) launch and more than 8 columns
    g.quantize_q8_1(0x1000, 0x20000, k, k, 1)
    ctx.flush()
    assert ctx.stats()["native_launches"] == 13
    ctx.flush()  # nothing held: no-op
    g.quantize_q8_1(0x1000, 0x20000, k, k, 1)
    args = cfi.KernelArgs([("ptr", 0)])
    assert ctx.launch(None, (1, 1, 1), (32, 1, 1), args) == 0
    s = ctx.stats()
    assert s["native_launches"] == 14 and s["stock_launches"] == 1
    g.quantize_q8_1(0x1000, 0x20000, k, k, 9)  # launched at once
    assert ctx.stats()["native_launches"] == 15
    ctx.close()


def test_quantize_is_not_deferred_without_the_flag():
    ctx, g = fake_caller()
    g.quantize_q8_1(0x1000, 0x20000, 2048, 2048, 1)
    assert ctx.stats()["native_launches"] == 1
    g.mmvq(cfi.Q4_K, 1, 0x100000, 0x20000, 0x300000, 2048, 8192)
    assert ctx.stats()["native_launches"] == 2 and ctx.stats()["fused_q8_1"] == 0
