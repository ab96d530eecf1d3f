"""The q4 projections either side of the attention path against the oracle:
kernels/matmul_nbits_sg.wgsl (nwd_q4_gemv), the fused q/k/v + kv_append
(nwd_q4_qkv_append) and one full engine attention layer step
(engine.AttentionLayer: runtime.js:321-335, :385-394)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from devutil import bits, to_dev, vals

pytestmark = pytest.mark.gpu


def _weights(ops, oracle, n, n_blocks, seed):
    b, s, z = oracle.q4_weights(n, n_blocks, seed)
    w = ops.Q4Weights(torch.from_numpy(b.view(np.int32)).cuda(), torch.from_numpy(s).cuda(),
                      torch.from_numpy(z.view(np.int32)).cuda())
    return w, (b, s, z)


def _act(oracle, k, seed):
    return oracle.f16_bits_to_f32(oracle.normal_f16(k, seed))


def _close_f32(got, ref, what):
    # f32 sums of K products in a different order: within 1e-5 of the output scale
    tol = 1e-5 * max(float(np.abs(ref).max()), 1.0)
    err = float(np.abs(got - ref).max())
    assert err <= tol, f"{what}: max |err| {err:.3e} > {tol:.3e}"


@pytest.mark.parametrize("K,N,epilogue", [
    (3136, 5120, 0),    # q_proj (hidden -> 40 x 128)
    (3136, 1024, 0),    # k_proj / v_proj
    (5120, 3136, 0),    # o_proj
    (3136, 12544, 1),   # MLP up with relu2 (matmul_nbits_sg.wgsl:76-79)
    (12544, 3136, 0),   # MLP down
    (96, 7, 0),         # ragged: N not a multiple of the column group
    (32, 33, 1),        # one block: only one warp of the CTA has work
    (14080, 40, 2),     # the largest K
])
def test_q4_gemv_vs_oracle(ops, oracle, K, N, epilogue):
    w, (b, s, z) = _weights(ops, oracle, N, K // 32, seed=K + N)
    a = _act(oracle, K, seed=7 + K)
    h = _act(oracle, N, seed=9)
    y = torch.from_numpy(h.copy()).cuda()
    ops.q4_gemv(torch.from_numpy(a).cuda(), w, y=y, epilogue=epilogue)
    ref = oracle.q4_gemv(a, b, s, z, epilogue=epilogue, y=h)
    _close_f32(y.cpu().numpy(), ref, f"K={K} N={N} epilogue={epilogue}")


def test_q4_gemv_residual_and_f16_activations(ops, oracle):
    """o_proj fed by the fp16 attention output, added into the residual stream
    (kernels/add.wgsl fused as epilogue 2)."""
    K, N = 5120, 3136
    w, (b, s, z) = _weights(ops, oracle, N, K // 32, seed=3)
    a16 = oracle.normal_f16(K, 4)
    h = _act(oracle, N, seed=5)
    y = torch.from_numpy(h.copy()).cuda()
    ops.q4_gemv(to_dev(a16, (K,)), w, y=y, epilogue=2)
    ref = oracle.q4_gemv(oracle.f16_bits_to_f32(a16), b, s, z, epilogue=2, y=h)
    _close_f32(y.cpu().numpy(), ref, "o_proj + residual")


def test_q4_gemv_rejects_bad_shapes(ops, oracle):
    w, _ = _weights(ops, oracle, 8, 2, seed=1)
    a = torch.zeros(63, device="cuda")
    with pytest.raises(ops.NwdError, match="32 \\* n_blocks"):
        ops.q4_gemv(a, w)
    with pytest.raises(ops.NwdError, match="exceeds 14080"):
        ops.q4_gemv(torch.zeros(441 * 32, device="cuda"), _weights(ops, oracle, 8, 441, seed=2)[0])
    # the activations are copied in 16-byte pieces
    with pytest.raises(ops.NwdError, match="16-byte aligned"):
        ops.q4_gemv(torch.zeros(65, device="cuda")[1:], _weights(ops, oracle, 8, 2, seed=1)[0])


@pytest.mark.parametrize("K,nh,nkv,hd,cap,seq", [
    (3136, 40, 8, 128, 256, 37),   # the model's attention layer
    (96, 3, 1, 40, 16, 15),        # column tiles straddling q / k / v, last cache row
])
def test_q4_qkv_append(ops, oracle, K, nh, nkv, hd, cap, seq):
    """q / k / v of one token in one launch, k and v written into cache row seq."""
    wq, hq = _weights(ops, oracle, nh * hd, K // 32, seed=11)
    wk, hk = _weights(ops, oracle, nkv * hd, K // 32, seed=12)
    wv, hv = _weights(ops, oracle, nkv * hd, K // 32, seed=13)
    h = _act(oracle, K, seed=14)
    kc = oracle.normal_f16(cap * nkv * hd, 15).reshape(cap, nkv, hd)
    vc = oracle.normal_f16(cap * nkv * hd, 16).reshape(cap, nkv, hd)
    dk, dv = to_dev(kc), to_dev(vc)
    q = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.q4_qkv_append(torch.from_numpy(h).cuda(), wq, wk, wv, q, dk, dv, seq)
    for got, (b, s, z), what in ((vals(q).reshape(-1), hq, "q"),
                                 (vals(dk)[seq].reshape(-1), hk, "k"),
                                 (vals(dv)[seq].reshape(-1), hv, "v")):
        ref = oracle.q4_gemv(h, b, s, z)
        # fp16 result of an f32 sum: within one fp16 rounding (and the sum's order)
        err = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
        assert float(err.max()) <= 1.2e-3, f"{what}: {float(err.max()):.3e}"
    # every other cache row untouched
    mask = np.ones(cap, bool)
    mask[seq] = False
    assert np.array_equal(bits(dk)[mask], kc[mask]) and np.array_equal(bits(dv)[mask], vc[mask])
    with pytest.raises(ops.NwdError, match=f"seq {cap} exceeds maxSeq {cap}"):
        ops.q4_qkv_append(torch.from_numpy(h).cuda(), wq, wk, wv, q, dk, dv, cap)


def test_attention_layer_steps(engine_mod, ops, oracle):
    """Six steps of one engine attention layer (q/k/v projections + append, attention,
    o_proj + residual) against the same composition on the oracle."""
    K, nh, nkv, hd, cap = 3136, 40, 8, 128, 256
    wq, hq = _weights(ops, oracle, nh * hd, K // 32, seed=21)
    wk, hk = _weights(ops, oracle, nkv * hd, K // 32, seed=22)
    wv, hv = _weights(ops, oracle, nkv * hd, K // 32, seed=23)
    wo, ho = _weights(ops, oracle, K, nh * hd // 32, seed=24)
    layer = engine_mod.AttentionLayer(wq, wk, wv, wo, nh, nkv, hd, cap)
    kc = np.zeros((cap, nkv, hd), np.uint16)
    vc = np.zeros((cap, nkv, hd), np.uint16)
    h = _act(oracle, K, seed=25)
    dh = torch.from_numpy(h.copy()).cuda()
    for t in range(6):
        hn = _act(oracle, K, seed=100 + t)
        layer.step(torch.from_numpy(hn).cuda(), dh)
        # the same step on the oracle, with the kernel's fp16 roundings
        q16 = oracle.f32_to_f16_bits(oracle.q4_gemv(hn, *hq))
        k16 = oracle.f32_to_f16_bits(oracle.q4_gemv(hn, *hk))
        v16 = oracle.f32_to_f16_bits(oracle.q4_gemv(hn, *hv))
        oracle.kv_append(k16, kc, t, nkv, hd)
        oracle.kv_append(v16, vc, t, nkv, hd)
        att = oracle.attention(q16, kc, vc, nh, nkv, hd, t + 1)
        o16 = oracle.f32_to_f16_bits(att)
        h = oracle.q4_gemv(oracle.f16_bits_to_f32(o16), *ho, epilogue=2, y=h)
        got = dh.cpu().numpy()
        # fp16 roundings of q/k/v/o may differ by an ulp between the two sides
        tol = 2e-3 * max(float(np.abs(h).max()), 1.0)
        err = float(np.abs(got - h).max())
        assert err <= tol, f"step {t}: {err:.3e} > {tol:.3e}"
        h = got.astype(np.float32)  # follow the kernel's residual stream
    assert layer.seq == 6
    assert layer.attn.workspace.check() == 0


def test_layers_with_weight_prefetch(engine_mod, ops, oracle):
    """engine.step_layers with the side-stream L2 weight prefetch gives bit-identical
    results to the same layers without it (the prefetch is only a hint), eager and
    captured in a CUDA graph."""
    K, nh, nkv, hd, cap, n_layers = 3136, 40, 8, 128, 256, 3

    def make():
        layers = []
        for i in range(n_layers):
            ws = [_weights(ops, oracle, n, nb, seed=300 + 4 * i + j)[0] for j, (n, nb) in
                  enumerate([(nh * hd, K // 32), (nkv * hd, K // 32), (nkv * hd, K // 32),
                             (K, nh * hd // 32)])]
            layer = engine_mod.AttentionLayer(*ws, nh, nkv, hd, cap)
            ops.fill_normal(layer.attn.k_cache, 70 + i)
            ops.fill_normal(layer.attn.v_cache, 80 + i)
            layer.attn.seq = 150
            layers.append(layer)
        return layers

    hn = torch.from_numpy(np.stack([_act(oracle, K, seed=400 + i) for i in range(n_layers)])).cuda()
    h0 = torch.from_numpy(_act(oracle, K, seed=450)).cuda()
    plain, pref = make(), make()
    h_plain, h_pref = h0.clone(), h0.clone()
    engine_mod.step_layers(plain, hn, h_plain)
    side = torch.cuda.Stream()
    engine_mod.step_layers(pref, hn, h_pref, side=side)
    torch.cuda.synchronize()
    assert torch.equal(h_plain, h_pref)
    for a, b in zip(plain, pref):
        assert torch.equal(a.attn.k_cache, b.attn.k_cache)
        assert torch.equal(a.attn.v_cache, b.attn.v_cache)
        assert a.seq == b.seq == 151
    # captured: fork and join of the side stream inside the graph
    stream = torch.cuda.Stream()
    for layer in pref:
        layer.attn.seq = 150
    for layer in plain:
        layer.attn.seq = 150
    h_plain.copy_(h0)
    engine_mod.step_layers(plain, hn, h_plain)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            engine_mod.step_layers(pref, hn, h_pref, side=side)
        h_pref.copy_(h0)
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(h_plain, h_pref)
    assert all(layer.attn.workspace.check() == 0 for layer in plain + pref)


def test_prefetch_l2_arguments(ops):
    """Ragged sizes and unaligned starts are accepted (the aligned interior is
    prefetched); more than 16 buffers or non-CUDA tensors are refused."""
    x = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    ops.prefetch_l2([x[1:], x[:7], x[16:4096 + 16]])
    ops.prefetch_l2([])
    torch.cuda.synchronize()
    with pytest.raises(ops.NwdError):
        ops.prefetch_l2([x] * 17)
    with pytest.raises(ValueError):
        ops.prefetch_l2([torch.zeros(4)])
