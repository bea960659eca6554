"""MoE top-k grouped expert FFN on the GPU vs the CPU oracle (W4A4 restatement of scripts/ref_forward.py:160-192).

Stage by stage:
  router    ids equal to the oracle's except at near-ties (8th/9th probability gap < 2e-6 relative), weights to 2e-4;
  dispatch  segment counts/starts, stable row order and the quantised dispatched rows bit-exact (segment padding
            rows are left unwritten: their products only reach outputs the epilogues never store);
  gate/up   the requantised intermediate agrees with the oracle's quantisation of the float64 h except where h is
            within rounding distance of a code boundary (>= 99.5% of codes equal, every difference one step);
  down      given the device's own intermediate, the combined output is within the W4A4 GEMM bar
            |Y - Yref| <= 1e-2 |Yref| + 1e-3 max|Yref|;
  end to end relative Frobenius error <= 2e-2 against the fully independent oracle.
Routing for the expert stages is taken from the device: at a near-tie between the 8th and 9th expert the fp32
logits of the device and the float64 oracle may pick different experts, which is not an expert-stage error."""
import numpy as np
import pytest
import torch

import native
import nvfp4_oracle as orc
from gpu_util import bf16_to_dev, gate_w4a4, require_gpu

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_problem(T, H, I, E, topk, seed=0):
    p = require_gpu()
    xb = orc.synth_bf16((T, H), 1.0, seed=seed)
    rb = orc.synth_bf16((E, H), 0.02, seed=seed + 1)
    experts = {}
    arena = p.MoeExperts(E, H, I)
    g1, g3, g2 = np.zeros(E, np.float32), np.zeros(E, np.float32), np.zeros(E, np.float32)
    for e in range(E):
        ex = {}
        for kind, shape, sd in [("gate", (I, H), 1000), ("up", (I, H), 2000), ("down", (H, I), 3000)]:
            wb = orc.synth_bf16(shape, 0.02, seed=seed + sd + e)
            g = orc.global_scale_from_amax(native.amax_bf16(wb))
            pk, sf = native.quantize_bf16(wb, g)
            ex[kind] = (pk, sf, g)
        experts[e] = ex
        arena.pack(e, _dev(ex["gate"][0]), _dev(ex["gate"][1]), _dev(ex["up"][0]), _dev(ex["up"][1]),
                   _dev(ex["down"][0]), _dev(ex["down"][1]))
        g1[e], g3[e], g2[e] = ex["gate"][2], ex["up"][2], ex["down"][2]
    arena.w1_gscale.copy_(torch.from_numpy(g1))
    arena.w3_gscale.copy_(torch.from_numpy(g3))
    arena.w2_gscale.copy_(torch.from_numpy(g2))
    g_in = orc.global_scale_from_amax(native.amax_bf16(xb))
    x = bf16_to_dev(xb)
    ws = p.moe_workspace(T, H, I, E, topk)
    return p, dict(xb=xb, x=x, rb=rb, proj=bf16_to_dev(rb), experts=experts, arena=arena, g_in=g_in, ws=ws,
                   T=T, H=H, I=I, E=E, topk=topk)


def route_and_calibrate(p, P):
    ids, w = p.moe_route(P["x"], P["proj"], P["topk"], P["ws"])
    h_amax = p.moe_calibrate(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]))
    torch.cuda.synchronize()
    g_h = np.array([orc.global_scale_from_amax(a) for a in h_amax.cpu().numpy()], np.float32)
    P["arena"].a2_gscale.copy_(torch.from_numpy(g_h))
    return ids, w, h_amax, g_h


def test_pack_expert_layout():
    p, P = make_problem(8, 256, 64, 4, 2)
    torch.cuda.synchronize()
    for e in range(4):
        ex = P["experts"][e]
        w13 = P["arena"].w13[e].cpu().numpy()
        for g in range(64 // 16):
            assert np.array_equal(w13[32 * g:32 * g + 16], ex["gate"][0][16 * g:16 * g + 16])
            assert np.array_equal(w13[32 * g + 16:32 * g + 32], ex["up"][0][16 * g:16 * g + 16])
        sf_rows = np.empty((128, 256 // 16), np.uint8)
        for g in range(4):
            sf_rows[32 * g:32 * g + 16] = ex["gate"][1][16 * g:16 * g + 16]
            sf_rows[32 * g + 16:32 * g + 32] = ex["up"][1][16 * g:16 * g + 16]
        assert np.array_equal(P["arena"].w13_scales[e].cpu().numpy(), orc.swizzle_scales(sf_rows, 128, 256))
        assert np.array_equal(P["arena"].w2[e].cpu().numpy(), ex["down"][0])
        assert np.array_equal(P["arena"].w2_scales[e].cpu().numpy(), orc.swizzle_scales(ex["down"][1], 256, 64))


@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("T,H,E", [(300, 512, 64), (300, 320, 64), (5, 128, 32)])
def test_router_matches_oracle(norm, T, H, E):
    topk = 8
    p = require_gpu()
    xb = orc.synth_bf16((T, H), 1.0, seed=3)
    rb = orc.synth_bf16((E, H), 0.02, seed=4)
    pes = (1.0 + 0.05 * np.random.default_rng(5).standard_normal(E)).astype(np.float32) if norm else None
    ws = p.moe_workspace(T, H, 64, E, topk)
    ids, w = p.moe_route(bf16_to_dev(xb), bf16_to_dev(rb), topk, ws,
                         per_expert_scale=_dev(pes) if norm else None, norm=norm)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    x = orc.bf16_bits_to_f32(xb).astype(np.float64)
    logits = x @ orc.bf16_bits_to_f32(rb).astype(np.float64).T
    if norm:
        logits = logits / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + 1e-6) * H ** -0.5
    w_ref, ids_ref = orc.route(logits.astype(np.float32), topk, pes)
    probs = np.sort(orc.softmax(logits.astype(np.float32)), axis=1)[:, ::-1]
    clear = (probs[:, topk - 1] - probs[:, topk]) > 2e-6 * probs[:, topk - 1] / probs[:, topk - 1].mean()
    got_ids, got_w = ids.cpu().numpy(), w.cpu().numpy()
    assert clear.mean() > 0.9
    assert np.array_equal(got_ids[clear], ids_ref[clear])
    assert np.allclose(got_w[clear], w_ref[clear], rtol=2e-4, atol=1e-5)
    if not norm:
        assert np.allclose(got_w.sum(1), 1.0, atol=1e-5)      # renormalised top-k weights


@pytest.mark.parametrize("T", [300, 1100])
def test_dispatch_plan_and_dispatched_rows_bit_exact(T):
    p, P = make_problem(T, 512, 128, 32, 8, seed=11)
    ids, w, _, _ = route_and_calibrate(p, P)
    out = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]))
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    v = p.moe_view(P["ws"], P["T"], P["H"], P["I"], P["E"], P["topk"])
    ids_np = ids.cpu().numpy()
    ref = orc.moe_dispatch_ref(ids_np, P["E"])
    assert int(v["m_tiles"].item()) == ref["m_tiles"]
    assert np.array_equal(v["seg_count"].cpu().numpy(), ref["seg_count"])
    assert np.array_equal(v["seg_start"].cpu().numpy(), ref["seg_start"])
    assert np.array_equal(v["dest"].cpu().numpy(), ref["dest"])
    rows = ref["m_tiles"] * 128
    real = ref["row_token"] >= 0          # segment padding rows are not written (the epilogues skip them)
    assert np.array_equal(v["row_token"].cpu().numpy()[:rows][real], ref["row_token"][real])
    te = v["tile_expert"].cpu().numpy()[:ref["m_tiles"]]
    assert np.array_equal(te, np.repeat(np.arange(P["E"]), (ref["seg_count"] + 127) // 128))
    # the dispatched rows are the oracle quantisation of x[token], bit for bit
    pk, sf = native.quantize_bf16(P["xb"], P["g_in"])
    a_codes = v["a_codes"].cpu().numpy()[:rows]
    a_sf = orc.unswizzle_scales(v["a_scales"].cpu().numpy(), v["rows"], P["H"])[:rows]
    assert np.array_equal(a_codes[real], pk[ref["row_token"][real]])
    assert np.array_equal(a_sf[real], sf[ref["row_token"][real]])
    assert np.all(np.isfinite(out.cpu().numpy()))


def _h_oracle_and_device(p, P, ids, w, g_h):
    v = p.moe_view(P["ws"], P["T"], P["H"], P["I"], P["E"], P["topk"])
    ref = orc.moe_dispatch_ref(ids, P["E"])
    rows = ref["m_tiles"] * 128
    h_codes = v["h_codes"].cpu().numpy()[:rows]
    h_sf = orc.unswizzle_scales(v["h_scales"].cpu().numpy(), v["rows"], P["I"])[:rows]
    return ref, h_codes, h_sf


def test_gate_up_requant_and_down_combine():
    p, P = make_problem(256, 512, 256, 32, 8, seed=21)
    ids, w, h_amax, g_h = route_and_calibrate(p, P)
    out = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]))
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    ids_np, w_np = ids.cpu().numpy(), w.cpu().numpy()
    ref, h_codes, h_sf = _h_oracle_and_device(p, P, ids_np, w_np, g_h)
    x = orc.bf16_bits_to_f32(P["xb"])
    # oracle h per expert (float64), quantised by the oracle
    full, hs = orc.moe_w4a4_ref(x, ids_np, w_np, P["experts"], P["g_in"], g_h)
    n_eq = n_all = 0
    override = {}
    for e, h in hs.items():
        r0, c = ref["seg_start"][e], ref["seg_count"][e]
        pk_ref, sf_ref, _ = orc.quantize_rows(h, g_h[e])
        dev_codes = orc.unpack_nibbles(h_codes[r0:r0 + c])
        ref_codes = orc.unpack_nibbles(pk_ref)
        n_eq += int((dev_codes == ref_codes).sum())
        n_all += dev_codes.size
        # calibration: device amax of h within fp32 accumulation error of the float64 amax
        assert abs(h_amax[e].item() - np.abs(h).max()) <= 1e-3 * np.abs(h).max()
        override[e] = (h_codes[r0:r0 + c], h_sf[r0:r0 + c])
    assert n_eq / n_all >= 0.995, n_eq / n_all
    # down + combine against the device's own intermediate: the W4A4 GEMM bar
    y_ref, _ = orc.moe_w4a4_ref(x, ids_np, w_np, P["experts"], P["g_in"], g_h, h_override=override)
    ok, msg = gate_w4a4(out.cpu().numpy(), y_ref)
    assert ok, msg
    # end to end against the independent oracle
    got = out.cpu().numpy().astype(np.float64)
    rel = np.linalg.norm(got - full) / np.linalg.norm(full)
    assert rel <= 2e-2, rel


@pytest.mark.parametrize("atomic", [False, True])
def test_accumulate_and_combine_modes(atomic):
    p, P = make_problem(64, 256, 64, 32, 4, seed=31)
    ids, w, _, _ = route_and_calibrate(p, P)
    base = torch.randn((64, 256), device="cuda", dtype=torch.float32)
    y0 = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]), atomic=atomic)
    y1 = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]), out=base.clone(),
                       accumulate=True, atomic=atomic)
    y2 = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]), atomic=not atomic)
    torch.cuda.synchronize()
    assert torch.allclose(y1, base + y0, rtol=1e-5, atol=1e-5)
    # the two combine modes agree up to the fp16 rounding of the deterministic mode's row buffer (2^-11 relative)
    assert torch.allclose(y0, y2, rtol=2e-3, atol=2e-3 * y2.abs().max().item())
    if not atomic:                                                 # the default combine is bit-reproducible
        y3 = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_gscale=float(P["g_in"]))
        torch.cuda.synchronize()
        assert torch.equal(y0, y3)


def test_cfg3_full_size_sampled_tokens():
    """cfg3: T=4096, H=2816, I=704, E=128, top-8; device routing; oracle on 48 sampled tokens (all their experts)
    using the device's intermediate for the down stage (W4A4 GEMM bar), dispatch invariants on all rows."""
    T, H, I, E, topk = 4096, 2816, 704, 128, 8
    p = require_gpu()
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = (torch.randn((T, H), generator=gen, device="cuda")).to(torch.bfloat16)
    proj = (torch.randn((E, H), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    arena = p.MoeExperts(E, H, I)
    experts = {}
    for e in range(E):
        mats = {}
        for kind, shape in [("gate", (I, H)), ("up", (I, H)), ("down", (H, I))]:
            wt = (torch.randn(shape, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
            amax = p.amax(wt)
            g = float(orc.global_scale_from_amax(amax.item()))
            pk, sf_swz = p.quantize(wt, gscale=g)
            mats[kind] = (pk, sf_swz, g, shape)
        sfl = {k: torch.from_numpy(orc.unswizzle_scales(m[1].cpu().numpy(), *m[3])).cuda() for k, m in mats.items()}
        arena.pack(e, mats["gate"][0], sfl["gate"], mats["up"][0], sfl["up"], mats["down"][0], sfl["down"])
        arena.w1_gscale[e], arena.w3_gscale[e], arena.w2_gscale[e] = mats["gate"][2], mats["up"][2], mats["down"][2]
        experts[e] = {k: (m[0].cpu().numpy(), sfl[k].cpu().numpy(), np.float32(m[2])) for k, m in mats.items()}
    ws = p.moe_workspace(T, H, I, E, topk)
    amax_x = p.amax(x)
    ids, w = p.moe_route(x, proj, topk, ws)
    h_amax = p.moe_calibrate(x, ids, w, arena, ws, in_amax=amax_x)
    torch.cuda.synchronize()
    g_h = np.array([orc.global_scale_from_amax(a) for a in h_amax.cpu().numpy()], np.float32)
    arena.a2_gscale.copy_(torch.from_numpy(g_h))
    out = p.moe_forward(x, ids, w, arena, ws, in_amax=amax_x)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    ids_np, w_np = ids.cpu().numpy(), w.cpu().numpy()
    ref = orc.moe_dispatch_ref(ids_np, E)
    v = p.moe_view(ws, T, H, I, E, topk)
    assert np.array_equal(v["dest"].cpu().numpy(), ref["dest"])
    assert np.array_equal(v["seg_count"].cpu().numpy(), ref["seg_count"])
    rng = np.random.default_rng(0)
    tokens = np.sort(rng.choice(T, 48, replace=False))
    rows_needed = ref["dest"].reshape(T, topk)[tokens].reshape(-1)
    h_codes = v["h_codes"].cpu().numpy()
    h_sf = orc.unswizzle_scales(v["h_scales"].cpu().numpy(), v["rows"], I)
    override = {}
    for e in np.unique(ids_np[tokens]):
        e = int(e)
        sel = np.nonzero(ids_np[tokens] == e)
        t_sel = tokens[sel[0]]
        order = np.lexsort((sel[1], t_sel))
        r = ref["dest"].reshape(T, topk)[t_sel[order], sel[1][order]]
        override[e] = (h_codes[r], h_sf[r])
    xf = orc.bf16_bits_to_f32(x.view(torch.int16).cpu().numpy().view(np.uint16))
    g_in = orc.global_scale_from_amax(amax_x.item())
    y_ref, _ = orc.moe_w4a4_ref(xf, ids_np, w_np, experts, g_in, g_h, h_override=override, tokens=tokens)
    ok, msg = gate_w4a4(out.cpu().numpy()[tokens], y_ref[tokens])
    assert ok, msg
    assert rows_needed.size == 48 * topk


def test_moe_forward_norm_fuses_input_rmsnorm():
    """nvfp4b_moe_forward_norm: the MoE input RMSNorm (x * rsqrt(mean(x^2) + eps) * w, the reference's
    pre_feedforward_layernorm_2) inside the quantise-dispatch.  The dispatched rows are the oracle quantisation of the
    float32-normalised rows (the device sums the squares in another order, so a value may sit on the other side of a
    rounding boundary in rare elements), and the layer matches the independent W4A4 oracle on the normalised input."""
    p, P = make_problem(96, 512, 128, 32, 8, seed=73)
    ids, w, _, g_h = route_and_calibrate(p, P)
    rng = np.random.default_rng(5)
    nw = orc.f32_to_bf16_bits((1.0 + 0.1 * rng.standard_normal(P["H"])).astype(np.float32))
    x2 = orc.rmsnorm(orc.bf16_bits_to_f32(P["xb"]), orc.bf16_bits_to_f32(nw), eps=1e-6)
    g_in = orc.global_scale_from_amax(np.float32(np.abs(x2).max()))
    out = p.moe_forward_norm(P["x"], ids, w, P["arena"], P["ws"], bf16_to_dev(nw), float(g_in), eps=1e-6)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    ids_np, w_np = ids.cpu().numpy(), w.cpu().numpy()
    v = p.moe_view(P["ws"], P["T"], P["H"], P["I"], P["E"], P["topk"])
    ref = orc.moe_dispatch_ref(ids_np, P["E"])
    rows = ref["m_tiles"] * 128
    real = ref["row_token"] >= 0
    pk, sf = native.quantize_f32(x2, g_in)
    a_codes = orc.unpack_nibbles(v["a_codes"].cpu().numpy()[:rows][real])
    a_sf = orc.unswizzle_scales(v["a_scales"].cpu().numpy(), v["rows"], P["H"])[:rows][real]
    want_codes = orc.unpack_nibbles(pk[ref["row_token"][real]])
    assert (a_codes == want_codes).mean() >= 0.999
    assert (a_sf == sf[ref["row_token"][real]]).mean() >= 0.999
    full, _ = orc.moe_w4a4_ref(x2, ids_np, w_np, P["experts"], g_in, g_h)
    got = out.cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - full) / np.linalg.norm(full) <= 2e-2


def test_moe_forward_norm_rejects_dynamic_scale():
    p, P = make_problem(8, 256, 64, 4, 2, seed=79)
    nw = bf16_to_dev(orc.f32_to_bf16_bits(np.ones(256, np.float32)))
    ids = torch.zeros((8, 2), dtype=torch.int32, device="cuda")
    ids[:, 1] = 1
    w = torch.full((8, 2), 0.5, device="cuda")
    with pytest.raises(p.NvFp4Error):
        p.moe_forward_norm(P["x"], ids, w, P["arena"], P["ws"], nw, 0.0)


@pytest.mark.parametrize("T,E,topk,norm,chain", [(512, 32, 8, False, True), (300, 64, 6, True, False),
                                                 (77, 32, 4, False, True), (1100, 32, 8, True, True)])
def test_moe_layer_router_fused_equals_route_then_forward(T, E, topk, norm, chain):
    """nvfp4b_moe_layer (router top-k fused with the dispatch ranking, seven launches) gives exactly what
    nvfp4b_moe_route followed by nvfp4b_moe_forward(_chain) gives: ids, weights, out, and the chained bf16 input and
    amax -- also for topk values that do not divide 256 (a block ranks the chunk of its own tokens' assignments)."""
    p, P = make_problem(T, 512, 128, E, topk, seed=83 + T)
    route_and_calibrate(p, P)
    rng = np.random.default_rng(T)
    pes = _dev((1.0 + 0.05 * rng.standard_normal(E)).astype(np.float32)) if norm else None
    amax = p.amax(P["x"])
    base = torch.randn((T, 512), device="cuda")
    ids_r, w_r = p.moe_route(P["x"], P["proj"], topk, P["ws"], per_expert_scale=pes, norm=norm)
    xn_r, an_r = (torch.empty_like(P["x"]), torch.zeros(1, device="cuda")) if chain else (None, None)
    out_r = p.moe_forward(P["x"], ids_r, w_r, P["arena"], P["ws"], in_amax=amax, out=base.clone(), accumulate=True,
                          x_next=xn_r, amax_next=an_r)
    ws2 = p.moe_workspace(T, 512, 128, E, topk)
    ids, w = torch.full_like(ids_r, -7), torch.full_like(w_r, float("nan"))
    xn, an = (torch.empty_like(P["x"]), torch.full((1,), 5.0, device="cuda")) if chain else (None, None)
    out = p.moe_layer(P["x"], P["proj"], topk, P["arena"], ws2, ids=ids, weights=w, per_expert_scale=pes, norm=norm,
                      in_amax=amax, out=base.clone(), accumulate=True, x_next=xn, amax_next=an)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    assert torch.equal(ids, ids_r) and torch.equal(w, w_r)
    assert torch.equal(out, out_r)
    if chain:
        assert torch.equal(xn, xn_r) and an.item() == an_r.item()
    v1 = p.moe_view(P["ws"], T, 512, 128, E, topk)
    v2 = p.moe_view(ws2, T, 512, 128, E, topk)
    assert torch.equal(v1["dest"], v2["dest"])            # the same rows, by either ranking
