"""GPU parity of the small ops against the CPU oracle, through the C ABI.

Stated tolerances: RMSNorm outputs are bf16 and may differ by one bf16 ulp where the GPU's
tree-ordered sum of squares rounds differently (<= 1 % of elements); the fused Q8_0
quantization of whatever bf16 values the GPU produced is bit-exact. RoPE tables and the
embedding gather are bit-exact. Attention and SiLU use expf and tree reductions: relative
error <= 2e-5 of the row's max |value|.
"""
import numpy as np
import pytest

from test_gpu_q8 import H, T

pytestmark = pytest.mark.gpu


def bf16_ulp_diff(a_bits, b_bits):
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # map sign-magnitude to a monotone integer line
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), 0x8000 + a)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + b)
    return np.abs(a - b)


@pytest.mark.parametrize("dim", [128, 1024, 4096, 5120])
@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_rmsnorm_and_fused_quant(ctx, lq8_lib, oracle, rng, dim, src):
    import torch
    rows = 6
    x = (rng.standard_normal((rows, dim)) * 2).astype(np.float32)
    if src == "bf16":
        x = oracle.f32_to_bf16(x)
    w = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(dim)).astype(np.float32))
    out = torch.empty((rows, dim), dtype=torch.int16, device="cuda")
    xq = torch.empty((rows, dim), dtype=torch.int8, device="cuda")
    xd = torch.empty((rows, dim // 32), dtype=torch.int16, device="cuda")
    dt = lq8_lib.DTYPE_F32 if src == "f32" else lq8_lib.DTYPE_BF16
    xt, wt = T(x), T(w)  # keep the device copies alive across the call
    ctx.call("lq_rmsnorm", xt.data_ptr(), dt, rows, dim, wt.data_ptr(), 1e-6, out.data_ptr(),
             xq.data_ptr(), xd.data_ptr())
    ctx.synchronize()
    got = H(out, np.uint16)
    ref = oracle.rmsnorm(x, w, 1e-6)
    diff = bf16_ulp_diff(got, ref)
    assert diff.max() <= 1 and (diff > 0).mean() <= 0.01
    oq, od = oracle.q8_0_quantize(got)
    assert np.array_equal(H(xq), oq) and np.array_equal(H(xd, np.uint16), od)


def test_rope_tables_bit_exact(ctx, lq8_lib, oracle):
    import torch
    c = torch.empty((300, 64), dtype=torch.float32, device="cuda")
    s = torch.empty_like(c)
    ctx.call("lq_rope_tables", 128, 300, 1e6, c.data_ptr(), s.data_ptr())
    oc, os_ = oracle.rope_tables(128, 300, 1e6)
    assert np.array_equal(H(c), oc) and np.array_equal(H(s), os_)


def _qk_ref(oracle, qkv, B, L, Hq, Hkv, qn, kn, pos0, ct, st):
    D = 128
    qkv = qkv.reshape(B, L, Hq + 2 * Hkv, D)
    q = np.zeros((B, Hq, L, D), np.float32)
    k = np.zeros((B, Hkv, L, D), np.float32)
    for b in range(B):
        for h in range(Hq):
            nb = oracle.rmsnorm(qkv[b, :, h, :].copy(), qn, 1e-6)
            q[b, h] = oracle.rope_apply(oracle.bf16_to_f32(nb)[None], pos0, ct, st)[0]
        for h in range(Hkv):
            nb = oracle.rmsnorm(qkv[b, :, Hq + h, :].copy(), kn, 1e-6)
            k[b, h] = oracle.rope_apply(oracle.bf16_to_f32(nb)[None], pos0, ct, st)[0]
    v = qkv[:, :, Hq + Hkv:, :].transpose(0, 2, 1, 3)
    return q, k, v


@pytest.mark.parametrize("B,L,pos0", [(1, 1, 0), (2, 1, 37), (1, 7, 0), (3, 5, 9)])
def test_qk_norm_rope_kv(ctx, lq8_lib, oracle, rng, B, L, pos0):
    import torch
    Hq, Hkv, D, ctx_max = 8, 2, 128, 64
    qkv = (rng.standard_normal((B * L, (Hq + 2 * Hkv) * D)) * 3).astype(np.float32)
    qn = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32))
    kn = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32))
    ct, st = oracle.rope_tables(D, ctx_max, 1e6)
    q_out = torch.zeros((B, Hq, L, D), dtype=torch.float32, device="cuda")
    kc = torch.zeros((B, Hkv, ctx_max, D), dtype=torch.float32, device="cuda")
    vc = torch.zeros_like(kc)
    keep = [T(a) for a in (qkv, qn, kn, ct, st)]
    ctx.call("lq_qk_norm_rope_kv", keep[0].data_ptr(), B, L, Hq, Hkv, D, keep[1].data_ptr(), keep[2].data_ptr(),
             1e-6, keep[3].data_ptr(), keep[4].data_ptr(), pos0, None, q_out.data_ptr(), kc.data_ptr(),
             vc.data_ptr(), ctx_max)
    ctx.synchronize()
    q, k, v = _qk_ref(oracle, qkv, B, L, Hq, Hkv, qn, kn, pos0, ct, st)
    gq, gk, gv = H(q_out), H(kc)[:, :, pos0:pos0 + L], H(vc)[:, :, pos0:pos0 + L]
    np.testing.assert_allclose(gq, q, rtol=0, atol=2e-2 * np.abs(q).max())  # 1 bf16 ulp of the norm
    assert np.mean(gq == q) > 0.98
    np.testing.assert_allclose(gk, k, rtol=0, atol=2e-2 * np.abs(k).max())
    assert np.array_equal(gv, v)
    assert not H(kc)[:, :, :pos0].any() and not H(kc)[:, :, pos0 + L:].any()


@pytest.mark.parametrize("B,L,pos0,ctx_max", [(1, 1, 0, 64), (2, 1, 200, 512), (1, 1, 2303, 2304),
                                              (1, 6, 0, 64), (2, 9, 130, 256)])
@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (32, 8), (8, 1)])
def test_attention_vs_oracle(ctx, lq8_lib, oracle, rng, B, L, pos0, ctx_max, Hq, Hkv):
    import torch
    D = 128
    G = Hq // Hkv
    T_ = pos0 + L
    q = rng.standard_normal((B, Hq, L, D)).astype(np.float32)
    kc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    vc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    kc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    vc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    out = torch.empty((B * L, Hq * D), dtype=torch.float32, device="cuda")
    xq = torch.empty((B * L, Hq * D), dtype=torch.int8, device="cuda")
    xd = torch.empty((B * L, Hq * D // 32), dtype=torch.int16, device="cuda")
    keep = [T(a) for a in (q, kc, vc)]
    ctx.call("lq_attention", keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), B, Hq, Hkv, L, pos0,
             None, ctx_max, D, out.data_ptr(), xq.data_ptr(), xd.data_ptr())
    ctx.synchronize()
    got = H(out).reshape(B, L, Hq, D)
    for b in range(B):
        for l in range(L):
            for h in range(Hq):
                ref = oracle.attend_row(q[b, h, l], kc[b, h // G, :T_], vc[b, h // G, :T_],
                                        masked=L > 1, causal_limit=pos0 + l)
                np.testing.assert_allclose(got[b, l, h], ref, rtol=0, atol=2e-5 * np.abs(ref).max())
    oq, od = oracle.q8_0_quantize(H(out))
    assert np.array_equal(H(xq), oq) and np.array_equal(H(xd, np.uint16), od)


@pytest.mark.parametrize("B,pos0,ctx_max,Hq,Hkv,dev_pos", [(8, 1030, 2048, 64, 8, True), (1, 0, 64, 32, 8, False),
                                                        (3, 63, 128, 16, 8, True), (5, 64, 256, 32, 4, False),
                                                        (2, 4095, 4096, 8, 1, True), (8, 700, 1024, 32, 8, False)])
def test_attention_decode_stream_vs_oracle(ctx, lq8_lib, oracle, rng, monkeypatch, B, pos0, ctx_max, Hq, Hkv,
                                           dev_pos):
    """The streamed decode attention (LQ_ATT_STREAM=1): the 32-key chunks of every (row, kv head)
    pair dealt over one CTA per SM through a bulk-copy ring, an online softmax over a CTA's
    chunks of a pair, and the pieces of a pair merged by the CTA that completes it. Every row
    against the oracle (the position also read from device memory, as the graph-replay decode
    does), the same bits on a second call, the Q8_0 output the quantization of the f32 output,
    and within the same bound of the chunk kernel (the default)."""
    import torch
    D = 128
    G = Hq // Hkv
    T_ = pos0 + 1
    q = rng.standard_normal((B, Hq, 1, D)).astype(np.float32)
    kc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    vc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    kc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    vc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    keep = [T(a) for a in (q, kc, vc)]
    pos_t = torch.tensor([pos0], dtype=torch.int32, device="cuda")

    def run():
        out = torch.full((B, Hq * D), float("nan"), dtype=torch.float32, device="cuda")
        xq = torch.empty((B, Hq * D), dtype=torch.int8, device="cuda")
        xd = torch.empty((B, Hq * D // 32), dtype=torch.int16, device="cuda")
        ctx.call("lq_attention", keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), B, Hq, Hkv, 1,
                 0 if dev_pos else pos0, pos_t.data_ptr() if dev_pos else None, ctx_max, D, out.data_ptr(),
                 xq.data_ptr(), xd.data_ptr())
        ctx.synchronize()
        return H(out), H(xq), H(xd, np.uint16)

    monkeypatch.setenv("LQ_ATT_STREAM", "1")
    got = run()
    again = run()
    for a, r in zip(got, again):
        assert np.array_equal(a.view(np.uint8), r.view(np.uint8))
    out = got[0].reshape(B, Hq, D)
    for b in range(B):
        for h in range(Hq):
            want = oracle.attend_row(q[b, h, 0], kc[b, h // G, :T_], vc[b, h // G, :T_], masked=False,
                                     causal_limit=pos0)
            np.testing.assert_allclose(out[b, h], want, rtol=0, atol=2e-5 * np.abs(want).max())
    oq, od = oracle.q8_0_quantize(got[0])
    assert np.array_equal(got[1], oq) and np.array_equal(got[2], od)
    monkeypatch.delenv("LQ_ATT_STREAM")
    ref = run()[0].reshape(B, Hq, D)
    np.testing.assert_allclose(out, ref, rtol=0, atol=4e-5 * np.abs(ref).max())


@pytest.mark.parametrize("B,L,pos0,ctx_max,dev_pos", [(8, 1, 1030, 2048, True), (3, 1, 63, 128, True),
                                                      (2, 1, 64, 256, False), (1, 1, 4095, 4096, True),
                                                      (2, 5, 60, 128, True), (1, 11, 0, 64, False)])
@pytest.mark.parametrize("Hq,Hkv", [(64, 8), (32, 8), (16, 8), (8, 8), (24, 8), (56, 8)])
def test_attention_chunk_bulk_vs_oracle(ctx, lq8_lib, oracle, rng, monkeypatch, B, L, pos0, ctx_max, Hq, Hkv,
                                        dev_pos):
    """The ring kernel of batched decode rows and short prefills: per (row, kv head) a few CTAs,
    each streaming its range of 32-position sub-chunks through a two-stage ring (K and V rows by
    bulk copies; the rows before the step's positions requested before the preceding kernel is
    waited on), scores and P.V as 3xTF32 tensor-core products (default) or f32 FMAs
    (LQ_ATT_FMA=1), an online softmax, one partial per range merged per query head by the merge
    kernel. Every row against the oracle (the position also from device memory, as graph replays
    pass it), ranges whose new rows start mid-sub-chunk or fill it, every group size 1..8 incl.
    the generic ones, the same bits on a second call, the Q8_0 output the quantization of the
    f32 output; the FMA variant and the cp.async chunk kernel (LQ_ATT_CP=1) within the same
    bound."""
    import torch
    D = 128
    G = Hq // Hkv
    T_ = pos0 + L
    q = rng.standard_normal((B, Hq, L, D)).astype(np.float32)
    kc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    vc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    kc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    vc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    keep = [T(a) for a in (q, kc, vc)]
    pos_t = torch.tensor([pos0], dtype=torch.int32, device="cuda")

    def run():
        out = torch.full((B * L, Hq * D), float("nan"), dtype=torch.float32, device="cuda")
        xq = torch.empty((B * L, Hq * D), dtype=torch.int8, device="cuda")
        xd = torch.empty((B * L, Hq * D // 32), dtype=torch.int16, device="cuda")
        ctx.call("lq_attention", keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), B, Hq, Hkv, L,
                 0 if dev_pos else pos0, pos_t.data_ptr() if dev_pos else None, ctx_max, D, out.data_ptr(),
                 xq.data_ptr(), xd.data_ptr())
        ctx.synchronize()
        return H(out), H(xq), H(xd, np.uint16)

    got = run()
    again = run()
    for a, r in zip(got, again):
        assert np.array_equal(a.view(np.uint8), r.view(np.uint8))
    out = got[0].reshape(B, L, Hq, D)
    for b in range(B):
        for l in range(L):
            for h in range(Hq):
                want = oracle.attend_row(q[b, h, l], kc[b, h // G, :T_], vc[b, h // G, :T_], masked=L > 1,
                                         causal_limit=pos0 + l)
                np.testing.assert_allclose(out[b, l, h], want, rtol=0, atol=2e-5 * np.abs(want).max())
    oq, od = oracle.q8_0_quantize(got[0])
    assert np.array_equal(got[1], oq) and np.array_equal(got[2], od)
    monkeypatch.setenv("LQ_ATT_FMA", "1")
    fma = run()[0].reshape(B, L, Hq, D)
    for b in range(B):
        for l in range(L):
            for h in range(Hq):
                want = oracle.attend_row(q[b, h, l], kc[b, h // G, :T_], vc[b, h // G, :T_], masked=L > 1,
                                         causal_limit=pos0 + l)
                np.testing.assert_allclose(fma[b, l, h], want, rtol=0, atol=2e-5 * np.abs(want).max())
    monkeypatch.delenv("LQ_ATT_FMA")
    monkeypatch.setenv("LQ_ATT_CP", "1")
    ref = run()[0].reshape(B, L, Hq, D)
    np.testing.assert_allclose(out, ref, rtol=0, atol=4e-5 * np.abs(ref).max())


@pytest.mark.parametrize("B,L,pos0,ctx_max", [(1, 16, 0, 64), (2, 47, 0, 128), (1, 200, 70, 300),
                                              (2, 129, 5, 2304), (1, 2048, 0, 2304)])
@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (32, 8), (64, 8), (32, 4), (8, 8)])
def test_attention_prefill_tiles_vs_oracle(ctx, lq8_lib, oracle, rng, B, L, pos0, ctx_max, Hq, Hkv):
    """Prefill attention (L >= 16: tiles of 128 (position, head) rows, online softmax over
    64-key chunks): ragged last tiles, a prompt appended after cached positions, every GQA
    group size Qwen3 uses. Rows are checked against the oracle's full-row softmax (all rows
    for small cases, a seeded sample at L = 2048)."""
    import torch
    D = 128
    G = Hq // Hkv
    T_ = pos0 + L
    q = rng.standard_normal((B, Hq, L, D)).astype(np.float32)
    kc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    vc = np.zeros((B, Hkv, ctx_max, D), np.float32)
    kc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D)) * 1.5
    vc[:, :, :T_] = rng.standard_normal((B, Hkv, T_, D))
    out = torch.empty((B * L, Hq * D), dtype=torch.float32, device="cuda")
    xq = torch.empty((B * L, Hq * D), dtype=torch.int8, device="cuda")
    xd = torch.empty((B * L, Hq * D // 32), dtype=torch.int16, device="cuda")
    keep = [T(a) for a in (q, kc, vc)]
    ctx.call("lq_attention", keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), B, Hq, Hkv, L, pos0,
             None, ctx_max, D, out.data_ptr(), xq.data_ptr(), xd.data_ptr())
    ctx.synchronize()
    got = H(out).reshape(B, L, Hq, D)
    rows = [(b, l, h) for b in range(B) for l in range(L) for h in range(Hq)]
    if len(rows) > 3000:
        pick = rng.choice(len(rows), 400, replace=False)
        rows = [rows[i] for i in pick] + [(0, L - 1, Hq - 1), (B - 1, 0, 0)]
    for b, l, h in rows:
        ref = oracle.attend_row(q[b, h, l], kc[b, h // G, :T_], vc[b, h // G, :T_], masked=True,
                                causal_limit=pos0 + l)
        np.testing.assert_allclose(got[b, l, h], ref, rtol=0, atol=2e-5 * np.abs(ref).max())
    oq, od = oracle.q8_0_quantize(H(out))
    assert np.array_equal(H(xq), oq) and np.array_equal(H(xd, np.uint16), od)


@pytest.mark.parametrize("m,inter", [(1, 3072), (5, 768), (16, 12288)])
def test_silu_mul_and_quant(ctx, lq8_lib, oracle, rng, m, inter):
    import torch
    gu = (rng.standard_normal((m, 2 * inter)) * 3).astype(np.float32)
    h = torch.empty((m, inter), dtype=torch.float32, device="cuda")
    xq = torch.empty((m, inter), dtype=torch.int8, device="cuda")
    xd = torch.empty((m, inter // 32), dtype=torch.int16, device="cuda")
    gut = T(gu)
    ctx.call("lq_silu_mul", gut.data_ptr(), m, inter, h.data_ptr(), xq.data_ptr(), xd.data_ptr())
    ctx.synchronize()
    g, u = gu[:, :inter], gu[:, inter:]
    ref = np.array([[oracle.silu(a) for a in row] for row in g[:, :512]], np.float32) * u[:, :512]
    np.testing.assert_allclose(H(h)[:, :512], ref, rtol=2e-6, atol=1e-7)
    oq, od = oracle.q8_0_quantize(H(h))
    assert np.array_equal(H(xq), oq) and np.array_equal(H(xd, np.uint16), od)


def test_embedding_gather_and_bad_id(ctx, lq8_lib, oracle, rng):
    import torch
    V, Hd = 1000, 256
    table = oracle.f32_to_bf16(rng.standard_normal((V, Hd)).astype(np.float32))
    ids = np.array([0, 999, 17, 17, 500], np.int32)
    out = torch.empty((5, Hd), dtype=torch.float32, device="cuda")
    tt, it = T(table), T(ids)
    ctx.call("lq_embedding", tt.data_ptr(), V, Hd, it.data_ptr(), 5, out.data_ptr())
    ctx.synchronize()
    assert np.array_equal(H(out), oracle.bf16_to_f32(table[ids]))
    bad = T(np.array([3, 1000], np.int32))
    with pytest.raises(lq8_lib.LQ8Error):
        ctx.call("lq_embedding", tt.data_ptr(), V, Hd, bad.data_ptr(), 2, out.data_ptr())


def test_argmax_ties_to_last(ctx, lq8_lib, oracle, rng):
    import torch
    x = rng.standard_normal((4, 151936)).astype(np.float32)
    x[1, 5] = x[1, 77] = x[1, 151935] = 100.0   # tie -> last index
    x[2, :] = -1.0                               # all equal -> last index
    x[3, 0] = 50.0
    out = torch.empty(4, dtype=torch.int32, device="cuda")
    xt = T(x)
    ctx.call("lq_argmax", xt.data_ptr(), 4, 151936, out.data_ptr())
    ctx.synchronize()
    assert H(out).tolist() == [oracle.argmax(r) for r in x]
    assert H(out).tolist()[1:] == [151935, 151935, 0]


def test_add(ctx, lq8_lib, rng):
    import torch
    a = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000).astype(np.float32)
    out = torch.empty(1000, dtype=torch.float32, device="cuda")
    at, bt = T(a), T(b)
    ctx.call("lq_add", at.data_ptr(), bt.data_ptr(), 1000, out.data_ptr())
    ctx.synchronize()
    assert np.array_equal(H(out), a + b)
