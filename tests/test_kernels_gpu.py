"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""
import math

import pytest
import torch

from sparsecache_b200.config import get_model_config
from sparsecache_b200.models.weights import interleave_gate_up
from sparsecache_b200.rope import relocate_positions, rope_cos_sin, rope_table

pytestmark = pytest.mark.gpu


def _ext():
    from sparsecache_b200 import ops

    return ops.ext()


def _status_ok(dev):
    st = _ext().status(torch.empty(1, device=dev))
    assert int(st.item()) == 0, f"kernel reported bounded-wait timeout {int(st.item())}"


def _rel_err(out, ref):
    return ((out.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("mnk", [(1, 256, 64), (130, 512, 320), (300, 6144, 4096), (1000, 4096, 1024)])
def test_gemm_store(cuda_device, bn, mnk):
    M, N, K = mnk
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    out = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    _ext().gemm_store(a, w, out, bn)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    ref = a.float() @ w.float().T
    assert _rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("mnk", [(300, 4096, 14336), (200, 4096, 4096), (64, 1024, 1024)])
def test_gemm_split_k_residual(cuda_device, mnk):
    """Split-K (fp32 slice partials + ordered reduce) equals the single-pass GEMM within bf16 rounding."""
    M, N, K = mnk
    g = torch.Generator(device="cpu").manual_seed(M * 7 + K)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(cuda_device, torch.bfloat16)
    res = torch.randn(M, N, generator=g).to(cuda_device, torch.bfloat16)
    ref = res.float() + (a.float() @ w.float().T).to(torch.bfloat16).float()
    outs = {}
    for splits in (1, 2, 3, -1):
        out = res.clone()
        launched = _ext().gemm_residual(a, w, out, out, 256, splits)
        torch.cuda.synchronize()
        _status_ok(cuda_device)
        assert launched == (1 if splits == 1 else launched)
        assert _rel_err(out, ref) < 1e-2, splits
        outs[splits] = out
    st = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    assert _ext().gemm_store(a, w, st, 256, 3) == 2
    torch.cuda.synchronize()
    assert _rel_err(st, a.float() @ w.float().T) < 1e-2


@pytest.mark.parametrize("M,K,splits", [(300, 4096, 3), (300, 14336, -1), (257, 512, 1), (1000, 4096, 1)])
def test_gemm_residual_with_fused_norm(cuda_device, M, K, splits):
    """gemm_residual(..., norm_w, norm_out): the RMSNorm of the new rows (fused into the split-K reduce
    when it splits) is bit-identical to the RMSNorm kernel run on the stored rows."""
    ext = _ext()
    N = 4096
    g = torch.Generator(device="cpu").manual_seed(M + K)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(cuda_device, torch.bfloat16)
    res = torch.randn(M, N, generator=g).to(cuda_device, torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(N, generator=g)).to(cuda_device, torch.bfloat16)
    out, normed = res.clone(), torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    launched = ext.gemm_residual(a, w, out, out, 256, splits, norm_w=nw, eps=1e-5, norm_out=normed)
    assert launched == 2
    plain = res.clone()
    ext.gemm_residual(a, w, plain, plain, 256, splits)
    ref_norm = torch.empty_like(normed)
    ext.rmsnorm(plain, None, nw, 1e-5, ref_norm)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert torch.equal(out, plain)
    assert torch.equal(normed, ref_norm)


def test_gemm_residual_and_swiglu(cuda_device):
    M, K, F = 257, 512, 1024
    a = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(K, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    res = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    out = res.clone()
    _ext().gemm_residual(a, w, out, out, 256)  # in place
    torch.cuda.synchronize()
    ref = res.float() + (a.float() @ w.float().T).to(torch.bfloat16).float()
    assert _rel_err(out, ref) < 1e-2

    wg = (torch.randn(F, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(F, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    wgu = interleave_gate_up(wg, wu)
    act = torch.empty(M, F, device=cuda_device, dtype=torch.bfloat16)
    _ext().gemm_swiglu(a, wgu, act, 256)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    gate = (a.float() @ wg.float().T).to(torch.bfloat16)
    up = (a.float() @ wu.float().T).to(torch.bfloat16)
    ref = torch.nn.functional.silu(gate.float()).to(torch.bfloat16).float() * up.float()
    assert _rel_err(act, ref) < 2e-2


@pytest.mark.parametrize("M", [129, 300, 513, 1000])
def test_gemm_two_accumulator_tiles(cuda_device, M):
    """256-row tiles (two TMEM accumulators sharing each B k-block; a short last m-tile runs one)
    give the same bits as 128-row tiles for every epilogue, and match the fp32 reference."""
    ext = _ext()
    cfg = get_model_config("tiny128")
    g = torch.Generator(device="cpu").manual_seed(M)
    K, N = 1024, 1536
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.03).to(cuda_device, torch.bfloat16)
    res = torch.randn(M, N, generator=g).to(cuda_device, torch.bfloat16)
    nq, nkv, cap = 8, 2, M + 64
    wq = (torch.randn((nq + 2 * nkv) * 128, K, generator=g) * 0.03).to(cuda_device, torch.bfloat16)
    pos = torch.arange(M, device=cuda_device, dtype=torch.int32) + 3
    slot = torch.arange(M, device=cuda_device, dtype=torch.int32) + 5
    table = rope_table(cfg, 2048, cuda_device)

    def run_all():
        outs = {}
        o = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
        ext.gemm_store(a, w, o, 256, 1)
        outs["store"] = o
        r = res.clone()
        ext.gemm_residual(a, w, r, r, 256, 1)
        outs["residual"] = r
        r2 = res.clone()
        ext.gemm_residual(a, w, r2, r2, 256, 3)
        outs["residual_split3"] = r2
        act = torch.empty(M, N // 2, device=cuda_device, dtype=torch.bfloat16)
        ext.gemm_swiglu(a, w, act, 256)
        outs["swiglu"] = act
        kc = torch.zeros(nkv, cap, 128, device=cuda_device, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        q = torch.empty(M, nq * 128, device=cuda_device, dtype=torch.bfloat16)
        dev = torch.zeros(M, 2 * nkv, device=cuda_device)
        ext.gemm_qkv(a, wq, q, kc, vc, pos, slot, table, nq, nkv, dev, 3, 256)
        outs.update(q=q, k=kc, v=vc, dev=dev)
        torch.cuda.synchronize()
        _status_ok(cuda_device)
        return outs

    try:
        ext.set_gemm_rows_per_tile(128)
        ref128 = run_all()
        ext.set_gemm_rows_per_tile(256)
        got = run_all()
    finally:
        ext.set_gemm_rows_per_tile(0)
    for name in ref128:
        assert torch.equal(got[name], ref128[name]), name
    y = a.float() @ w.float().T
    assert _rel_err(got["store"], y) < 1e-2
    assert _rel_err(got["residual"], res.float() + y.to(torch.bfloat16).float()) < 1e-2
    assert _rel_err(got["residual_split3"], res.float() + y.to(torch.bfloat16).float()) < 1e-2


def _qkv_reference(a, w, cfg, pos, nq, nkv):
    y = a.float() @ w.float().T
    D = 128
    q = y[:, : nq * D].reshape(-1, nq, D)
    k = y[:, nq * D : (nq + nkv) * D].reshape(-1, nkv, D)
    v = y[:, (nq + nkv) * D :].reshape(-1, nkv, D)
    cos, sin = rope_cos_sin(cfg, pos.cpu(), device=a.device)
    cos, sin = cos[:, None, :], sin[:, None, :]

    def rot(x):
        return torch.cat((-x[..., 64:], x[..., :64]), dim=-1)

    return q * cos + rot(q) * sin, k * cos + rot(k) * sin, v


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("dev_mode", [0, 1, 2, 3, 6])
def test_gemm_qkv_rope_scatter_deviation(cuda_device, dev_mode, bn):
    cfg = get_model_config("tiny128")
    nq, nkv, K, M, cap = 4, 2, 512, 200, 600
    a = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn((nq + 2 * nkv) * 128, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    pos = torch.sort(torch.randperm(500)[:M]).values.to(torch.int32).to(cuda_device) + 7
    slot = torch.sort(torch.randperm(cap)[:M]).values.to(torch.int32).to(cuda_device)
    kc = torch.randn(nkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    vc = torch.randn(nkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    kc0, vc0 = kc.clone(), vc.clone()
    q_out = torch.empty(M, nq * 128, device=cuda_device, dtype=torch.bfloat16)
    table = rope_table(cfg, 1024, cuda_device)
    dev = torch.zeros(M, 2 * nkv, device=cuda_device) if dev_mode else None
    _ext().gemm_qkv(a, w, q_out, kc, vc, pos, slot, table, nq, nkv, dev, dev_mode, bn)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    q, k, v = _qkv_reference(a, w, cfg, pos, nq, nkv)
    assert _rel_err(q_out.reshape(M, nq, 128), q) < 1e-2
    sl = slot.long()
    assert _rel_err(kc[:, sl].transpose(0, 1), k) < 1e-2
    assert _rel_err(vc[:, sl].transpose(0, 1), v) < 1e-2
    untouched = torch.ones(cap, dtype=torch.bool, device=cuda_device)
    untouched[sl] = False
    assert torch.equal(kc[:, untouched], kc0[:, untouched])
    if dev_mode:
        kb = k.to(torch.bfloat16).float()
        vb = v.to(torch.bfloat16).float()
        dk = kb - kc0[:, sl].transpose(0, 1).float()
        dv = vb - vc0[:, sl].transpose(0, 1).float()
        f = (lambda x: x.abs()) if dev_mode & 4 else (lambda x: x.square())
        if dev_mode & 1:
            torch.testing.assert_close(dev[:, :nkv], f(dk).sum(-1), rtol=2e-2, atol=1e-1)
        if dev_mode & 2:
            torch.testing.assert_close(dev[:, nkv:], f(dv).sum(-1), rtol=2e-2, atol=1e-1)


def _attn_reference(q, kc, vc, qpos, kpos, n_heads):
    # q [R, H*128]; kc [Hkv, n, 128]
    R = q.shape[0]
    Hkv = kc.shape[0]
    G = n_heads // Hkv
    qh = q.float().reshape(R, n_heads, 128).transpose(0, 1)  # [H, R, D]
    k = kc.float().repeat_interleave(G, dim=0)
    v = vc.float().repeat_interleave(G, dim=0)
    s = qh @ k.transpose(1, 2) / math.sqrt(128)
    mask = kpos[None, :] <= qpos[:, None]
    s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return (p @ v).transpose(0, 1).reshape(R, n_heads * 128)


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("T,R", [(777, 150), (1676, 300), (65, 1), (129, 3), (4500, 120)])
@pytest.mark.parametrize("case", ["causal", "selective", "staged", "growing"])
def test_attention_prefill(cuda_device, case, T, R, split):
    """tcgen05 flash attention vs the fp32 reference: full causal rows, a sorted
    subset of rows over the whole cache (CacheBlend), staged key positions (a
    suffix at later global positions), and scores that grow along the keys so
    the lazily rescaled running max moves many times (the O-in-TMEM rescale).
    With ``split`` the kernel gets a workspace and splits the key tiles of
    small grids over several CTAs (fp32 partials + merge kernel)."""
    H, Hkv = 8, 2
    cap = T + 223
    g = torch.Generator(device="cpu").manual_seed(T * 7 + R + len(case))
    kc = torch.randn(Hkv, cap, 128, generator=g)
    vc = torch.randn(Hkv, cap, 128, generator=g)
    if case == "growing":
        kc[:, :T] *= torch.linspace(0.2, 3.0, T)[None, :, None]
    kc = kc.to(cuda_device, torch.bfloat16)
    vc = vc.to(cuda_device, torch.bfloat16)
    kpos = torch.arange(T, device=cuda_device, dtype=torch.int32)
    if case in ("causal", "growing"):
        rows = torch.arange(T, device=cuda_device, dtype=torch.int32)
        qpos = kpos.clone()
    else:
        rows = torch.sort(torch.randperm(T, generator=g)[:R]).values.to(torch.int32).to(cuda_device)
        qpos = kpos[rows.long()]
        if case == "staged":  # suffix placed at a later global position
            kpos = kpos.clone()
            kpos[-min(40, T // 2):] += 300
            qpos = kpos[rows.long()]
    qfull = torch.randn(T, H * 128, generator=g).to(cuda_device, torch.bfloat16)
    if case == "growing":
        qfull = (qfull.float() * 2.0).to(torch.bfloat16)
    out = torch.empty(rows.numel(), H * 128, device=cuda_device, dtype=torch.bfloat16)
    ws = None
    if split:
        ws = torch.full((4 * rows.numel() * H * 132,), float("nan"), device=cuda_device)
        n_split = _ext().attention_prefill_splits(rows.numel(), H, Hkv, T, ws.numel(), _ext().num_sms())
        if case not in ("causal", "growing") and (T, R) == (4500, 120):
            assert n_split > 1
    _ext().attention_prefill(
        qfull, rows, qpos, kc, vc, kpos if case == "staged" else None, T, H, 1 / math.sqrt(128), out, ws=ws
    )
    torch.cuda.synchronize()
    assert int(_ext().status(out).item()) == 0
    ref = _attn_reference(qfull[rows.long()], kc[:, :T], vc[:, :T], qpos.long(), kpos.long(), H)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M", [1, 5])
def test_attention_decode(cuda_device, M):
    H, Hkv, cap = 8, 2, 1200
    pos0 = 913
    kc = torch.randn(Hkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    vc = torch.randn(Hkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    q = torch.randn(M, H * 128, device=cuda_device).to(torch.bfloat16)
    pos = torch.tensor([pos0], device=cuda_device, dtype=torch.int32)
    n = pos0 + M
    kpos = torch.arange(n, device=cuda_device)
    qpos = pos0 + torch.arange(M, device=cuda_device)
    ref = _attn_reference(q, kc[:, :n], vc[:, :n], qpos, kpos, H)
    for splits in (1, 8, 16):  # cluster sizes, incl. CTAs whose chunk is past the last key
        out = torch.empty(M, H * 128, device=cuda_device, dtype=torch.bfloat16)
        _ext().attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), splits, out)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("hkv,G", [(2, 4), (1, 8)])
def test_attention_decode_batched_sequences(cuda_device, hkv, G):
    """One launch over B independent sequences (own position, own slot stride apart) equals one
    launch per sequence bit for bit, and the fp32 reference."""
    H, cap, B = hkv * G, 900, 5
    g = torch.Generator(device="cpu").manual_seed(11 + hkv)
    kc = torch.randn(B, hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16)
    vc = torch.randn(B, hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16)
    q = torch.randn(B, H * 128, generator=g).to(cuda_device, torch.bfloat16)
    positions = [37, 899, 400, 0, 511]
    pos_rows = torch.tensor(positions, device=cuda_device, dtype=torch.int32)
    out = torch.empty(B, H * 128, device=cuda_device, dtype=torch.bfloat16)
    stride = hkv * cap * 128
    for splits in (4, 8):
        _ext().attention_decode(q, kc[0], vc[0], pos_rows, H, 1 / math.sqrt(128), splits, out,
                                pos_rows=pos_rows, seq_stride=stride)
        torch.cuda.synchronize()
        for b, p in enumerate(positions):
            one = torch.empty(1, H * 128, device=cuda_device, dtype=torch.bfloat16)
            pos = torch.tensor([p], device=cuda_device, dtype=torch.int32)
            _ext().attention_decode(q[b:b + 1], kc[b], vc[b], pos, H, 1 / math.sqrt(128), splits, one)
            torch.cuda.synchronize()
            assert torch.equal(one, out[b:b + 1]), (splits, b)
            ref = _attn_reference(q[b:b + 1], kc[b, :, :p + 1], vc[b, :, :p + 1],
                                  torch.tensor([p], device=cuda_device), torch.arange(p + 1, device=cuda_device), H)
            torch.testing.assert_close(out[b:b + 1].float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("hkv,cap", [(1, 16384), (2, 12000), (4, 18000)])
def test_attention_decode_two_level_split(cuda_device, M, hkv, cap):
    """Several clusters per kv head (few kv heads / long contexts): the ticketed
    cross-cluster merge equals the reference, twice in a row (the tickets reset)."""
    G = 8 if hkv == 1 else 4
    H = hkv * G
    pos0 = cap - 40
    g = torch.Generator(device="cpu").manual_seed(cap + M)
    kc = torch.randn(hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16)
    vc = torch.randn(hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16)
    q = torch.randn(M, H * 128, generator=g).to(cuda_device, torch.bfloat16)
    pos = torch.tensor([pos0], device=cuda_device, dtype=torch.int32)
    n = pos0 + M
    ref = _attn_reference(q, kc[:, :n], vc[:, :n], pos0 + torch.arange(M, device=cuda_device),
                          torch.arange(n, device=cuda_device), H)
    ws = torch.zeros(hkv * 16 * 64 * 130, device=cuda_device)
    cnt = torch.zeros(hkv * 16, device=cuda_device, dtype=torch.int32)
    S = _ext().attention_decode_cluster(cap, hkv)
    outer = _ext().attention_decode_outer(cap, hkv, S, _ext().num_sms())
    assert S == 4 and outer > 1
    for _ in range(2):
        out = torch.empty(M, H * 128, device=cuda_device, dtype=torch.bfloat16)
        _ext().attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), S, out, ws=ws, counters=cnt)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
        assert int(cnt.sum()) == 0


@pytest.mark.parametrize("M", [1, 3])
@pytest.mark.parametrize("n_vis", [700, 5000])
def test_attention_decode_sparse_view_key_capacity(cuda_device, M, n_vis):
    """A small page view of a long cache: the split sized for the view's keys (key_capacity) and the
    split sized for the whole cache both equal the fp32 reference over the gathered keys."""
    hkv, G, cap = 8, 4, 40000
    H = hkv * G
    g = torch.Generator(device="cpu").manual_seed(n_vis + M)
    kc = torch.randn(hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16)
    vc = torch.randn(hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16)
    q = torch.randn(M, H * 128, generator=g).to(cuda_device, torch.bfloat16)
    p0 = cap - 64  # the query rows' own slots (their K/V already in the cache)
    vis = torch.sort(torch.randperm(p0, generator=g)[:n_vis]).values
    table = torch.cat((vis, torch.arange(p0, p0 + M))).to(torch.int32).to(cuda_device)
    view = torch.zeros(cap, dtype=torch.int32, device=cuda_device)
    view[: table.numel()] = table
    nv = torch.tensor([n_vis + M], dtype=torch.int32, device=cuda_device)
    pos = torch.tensor([p0], dtype=torch.int32, device=cuda_device)
    idx = table.long()
    ref = _attn_reference(q, kc[:, idx], vc[:, idx], n_vis + torch.arange(M, device=cuda_device),
                          torch.arange(n_vis + M, device=cuda_device), H)
    ws = torch.zeros(hkv * 16 * 64 * 130, device=cuda_device)
    cnt = torch.zeros(hkv * 16, device=cuda_device, dtype=torch.int32)
    outs = []
    for key_cap in (n_vis + M, 0):
        S = _ext().attention_decode_cluster(key_cap or cap, hkv)
        out = torch.empty(M, H * 128, device=cuda_device, dtype=torch.bfloat16)
        _ext().attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), S, out, page_table=view, page_shift=0,
                                n_virtual=nv, ws=ws, counters=cnt, key_capacity=key_cap)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
        assert int(cnt.sum()) == 0
        outs.append(out)
    with pytest.raises(RuntimeError):  # the key-count split is for paged views only
        _ext().attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), 8, outs[0], key_capacity=n_vis + M)


def _rms_ref(x, w, eps):
    xf = x.float()
    r = torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return (w.float() * (xf * r).to(torch.bfloat16).float())


@pytest.mark.parametrize("M", [1, 3, 8])
def test_gemv_variants(cuda_device, M):
    K, N = 1024, 768
    eps = 1e-5
    x = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device=cuda_device)).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    ext = _ext()
    out = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    ext.gemv_store(x, w, nw, eps, out)
    torch.cuda.synchronize()
    xn = _rms_ref(x, nw, eps).to(torch.bfloat16).float()
    assert _rel_err(out, xn @ w.float().T) < 1e-2

    res = torch.randn(M, N, device=cuda_device).to(torch.bfloat16)
    out2 = res.clone()
    ext.gemv_residual(x, w, None, eps, out2, out2)
    torch.cuda.synchronize()
    ref = res.float() + (x.float() @ w.float().T).to(torch.bfloat16).float()
    assert _rel_err(out2, ref) < 1e-2

    F = 512
    wg = (torch.randn(F, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(F, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    act = torch.empty(M, F, device=cuda_device, dtype=torch.bfloat16)
    ext.gemv_swiglu(x, interleave_gate_up(wg, wu), None, eps, act)
    torch.cuda.synchronize()
    g = (x.float() @ wg.float().T).to(torch.bfloat16).float()
    u = (x.float() @ wu.float().T).to(torch.bfloat16).float()
    ref = torch.nn.functional.silu(g).to(torch.bfloat16).float() * u
    assert _rel_err(act, ref) < 2e-2


def test_gemv_qkv_and_argmax(cuda_device):
    cfg = get_model_config("tiny128")
    nq, nkv, K, cap, V = 4, 2, 512, 300, 4096
    ext = _ext()
    x = torch.randn(1, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn((nq + 2 * nkv) * 128, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    kc = torch.zeros(nkv, cap, 128, device=cuda_device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(1, nq * 128, device=cuda_device, dtype=torch.bfloat16)
    pos = torch.tensor([123], device=cuda_device, dtype=torch.int32)
    table = rope_table(cfg, 1024, cuda_device)
    ext.gemv_qkv(x, w, None, 1e-5, q_out, kc, vc, pos, table, nq, nkv)
    torch.cuda.synchronize()
    q, k, v = _qkv_reference(x, w, cfg, pos, nq, nkv)
    assert _rel_err(q_out.reshape(1, nq, 128), q) < 1e-2
    assert _rel_err(kc[:, 123].unsqueeze(0), k) < 1e-2
    assert _rel_err(vc[:, 123].unsqueeze(0), v) < 1e-2

    lm = (torch.randn(V, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    emb = torch.randn(V, K, device=cuda_device).to(torch.bfloat16)
    grid = ext.gemv_argmax_grid(V)
    pv = torch.empty(8 * grid, device=cuda_device)
    pi = torch.empty(8 * grid, device=cuda_device, dtype=torch.int32)
    counter = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    tok = torch.empty(3, device=cuda_device, dtype=torch.int32)
    log = torch.zeros(4, device=cuda_device, dtype=torch.int32)
    gen = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    nxt = torch.empty(1, K, device=cuda_device, dtype=torch.bfloat16)
    pos2 = torch.tensor([10], device=cuda_device, dtype=torch.int32)
    xs = torch.randn(3, K, device=cuda_device).to(torch.bfloat16)
    ext.gemv_argmax(xs, lm, None, 1e-5, pv, pi, counter, tok, log, gen, emb, nxt, pos2)
    torch.cuda.synchronize()
    # the kernel takes the argmax of bf16-rounded logits (lowest index on ties): rows whose fp32
    # logit lies within two bf16 spacings of the maximum may round to a tie or swap order
    logits = (xs.float() @ lm.float().T)
    for m in range(3):
        top = logits[m].max()
        spacing = 2.0 ** (torch.floor(torch.log2(top.abs())) - 7)
        near = (logits[m] >= top - 2 * spacing).nonzero().flatten().tolist()
        assert int(tok[m]) in near, (int(tok[m]), near)
    assert int(gen.item()) == 1 and int(log[0]) == int(tok[2])
    assert int(pos2.item()) == 13
    assert int(counter.item()) == 0
    assert torch.equal(nxt[0], emb[int(tok[2])])


def test_rmsnorm_embedding_gather(cuda_device):
    ext = _ext()
    V, D = 1000, 512
    table = torch.randn(V, D, device=cuda_device).to(torch.bfloat16)
    ids = torch.randint(0, V, (77,), device=cuda_device, dtype=torch.int32)
    h = torch.empty(77, D, device=cuda_device, dtype=torch.bfloat16)
    ext.embedding(ids, table, h)
    assert torch.equal(h, table[ids.long()])
    w = (1 + 0.1 * torch.randn(D, device=cuda_device)).to(torch.bfloat16)
    rows = torch.tensor([5, 0, 76], device=cuda_device, dtype=torch.int32)
    out = torch.empty(3, D, device=cuda_device, dtype=torch.bfloat16)
    ext.rmsnorm(h, rows, w, 1e-5, out)
    torch.cuda.synchronize()
    ref = _rms_ref(h[rows.long()], w, 1e-5)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)
    g = torch.empty(3, D, device=cuda_device, dtype=torch.bfloat16)
    ext.gather_rows(h, rows, g)
    assert torch.equal(g, h[rows.long()])


@pytest.mark.parametrize("host_source", [False, True])
def test_compose_relocate(cuda_device, host_source):
    cfg = get_model_config("tiny128")
    L, Hkv, cap = 3, 2, 900
    lens = [37, 120, 64, 5]
    docs = []
    for n in lens:
        t = torch.randn(L, 2, Hkv, n, 128).to(torch.bfloat16)
        docs.append(t.pin_memory() if host_source else t.to(cuda_device))
    cache = torch.zeros(L, 2, Hkv, cap, 128, device=cuda_device, dtype=torch.bfloat16)
    table = rope_table(cfg, 2048, cuda_device)
    rows, offs, cursor = [], [0], 50
    for t, n in zip(docs, lens):
        ptr = t.data_ptr()
        rows.append([ptr & 0xFFFFFFFF, ptr >> 32, n, 0, cursor, cursor])
        offs.append(offs[-1] + n)
        cursor += n
    doc_t = torch.tensor(rows, dtype=torch.int64)
    doc_t = torch.where(doc_t >= 2**31, doc_t - 2**32, doc_t).to(torch.int32).to(cuda_device)
    off_t = torch.tensor(offs, dtype=torch.int32, device=cuda_device)
    _ext().compose_relocate(doc_t, off_t, offs[-1], 0, L, L, cache, Hkv, table)
    torch.cuda.synchronize()
    cursor = 50
    for t, n in zip(docs, lens):
        src = t.to(cuda_device)
        for layer in range(L):
            k = src[layer, 0].unsqueeze(0)
            ref_k = relocate_positions(cfg, k, torch.arange(n), torch.arange(cursor, cursor + n))[0]
            got_k = cache[layer, 0, :, cursor : cursor + n]
            torch.testing.assert_close(got_k.float(), ref_k.float(), rtol=1e-2, atol=2e-2)
            assert torch.equal(cache[layer, 1, :, cursor : cursor + n], src[layer, 1])
        cursor += n


@pytest.mark.parametrize("keep_prefix", [True, False])
def test_cacheblend_select(cuda_device, keep_prefix):
    ext = _ext()
    T, nkv, doc_begin, doc_end = 3000, 8, 32, 2950
    dev = torch.rand(T, 2 * nkv, device=cuda_device)
    n_doc = doc_end - doc_begin
    k = math.ceil(0.15 * n_doc)
    active = torch.empty(T, device=cuda_device, dtype=torch.int32)
    n_active = torch.empty(1, device=cuda_device, dtype=torch.int32)
    scores = torch.empty(T, device=cuda_device)
    ck = torch.zeros(1, device=cuda_device, dtype=torch.int64)
    ext.cacheblend_select(dev, nkv, 2, T, doc_begin, doc_end, k, keep_prefix, active, n_active, scores, ck)
    torch.cuda.synchronize()
    s = dev[doc_begin:doc_end, nkv:].sum(-1)
    sel = torch.topk(s, k).indices + doc_begin
    parts = [sel, torch.arange(doc_end, T, device=cuda_device)]
    if keep_prefix:
        parts.insert(0, torch.arange(0, doc_begin, device=cuda_device))
    expect = torch.cat(parts).sort().values
    n = int(n_active.item())
    assert n == expect.numel()
    assert torch.equal(active[:n].long(), expect)
    ss = sel.sort().values
    assert int(ck.item()) == int((ss * torch.arange(1, k + 1, device=cuda_device)).sum())


def test_bounded_wait_times_out_then_fails_fast(cuda_device):
    """A flag nothing sets: the wait records a time-out and returns; later waits on the
    same status return at once; the context stays usable (no GPU fault involved)."""
    import time

    ext = _ext()
    flags = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ext.wait_flag(flags, 1, 1, int(2e6), status)  # 2 ms limit
    torch.cuda.synchronize()
    assert int(status.item()) != 0
    t0 = time.perf_counter()
    ext.wait_flag(flags, 2, 1, int(10e9), status)  # would wait 10 s without fail-fast
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    status.zero_()
    flags[2] = 5
    ext.wait_flag(flags, 2, 5, int(1e9), status)  # satisfied flag, clean status
    torch.cuda.synchronize()
    assert int(status.item()) == 0


@pytest.mark.parametrize("M", [3, 5, 8])
def test_gemv_wide_k_reads_x_from_global(cuda_device, M):
    """M * K * 2 bytes above the shared-memory budget (verify rows x a 28672-wide FFN):
    x is read from global memory; rows are independent of M."""
    K, N = 28672, 1024
    x = (torch.randn(M, K, device=cuda_device) * 0.1).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device) * 0.02).to(torch.bfloat16)
    res = torch.randn(M, N, device=cuda_device).to(torch.bfloat16)
    out = res.clone()
    ext = _ext()
    ext.gemv_residual(x, w, None, 1e-5, out, out)
    one = res[:1].clone()
    ext.gemv_residual(x[:1].contiguous(), w, None, 1e-5, one, one)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    ref = res.float() + (x.float() @ w.float().T).to(torch.bfloat16).float()
    assert _rel_err(out, ref) < 1e-2
    assert torch.equal(out[:1], one)  # the row does not depend on how many rows share the launch


def test_lse_gather_forward_backward(cuda_device):
    """Row log-sum-exp + logit gathers and the logits gradient against fp32 autograd."""
    from sparsecache_b200.ops.lm_loss import FrozenLMHead, lse_gather, lse_gather_reference

    torch.manual_seed(0)
    R, V, G = 300, 32000, 65
    logits = (torch.randn(R, V, device=cuda_device) * 3).to(torch.bfloat16)
    ids = torch.randint(0, V, (R, G), device=cuda_device, dtype=torch.int32)
    ids[::7, 5:9] = -1
    ids[:, 3] = ids[:, 0]  # duplicate ids add up
    a = torch.randn(R, device=cuda_device)
    b = torch.randn(R, G, device=cuda_device)
    x = logits.clone().requires_grad_(True)
    lse, z = lse_gather(x, ids)
    ((a * lse).sum() + (b * z).sum()).backward()
    xr = logits.float().clone().requires_grad_(True)
    lse_r, z_r = lse_gather_reference(xr, ids)
    ((a * lse_r).sum() + (b * z_r).sum()).backward()
    torch.cuda.synchronize()
    assert _rel_err(lse, lse_r) < 1e-5 and torch.equal(z, z_r.detach())
    assert _rel_err(x.grad, xr.grad) < 2e-2
    # fused LM head: feats -> (lse, z), gradient into feats through the frozen head
    d = 512
    w = (torch.randn(4096, d, device=cuda_device) * 0.05).to(torch.bfloat16)
    head = FrozenLMHead(w)
    f = torch.randn(R, d, device=cuda_device).to(torch.bfloat16).requires_grad_(True)
    ids2 = ids.clamp_max(4095)
    lse2, z2 = head.lse_gather(f, ids2)
    ((a * lse2).sum() + (b * z2).sum()).backward()
    fr = f.detach().float().clone().requires_grad_(True)
    lse2r, z2r = lse_gather_reference(fr @ w.float().t(), ids2)
    ((a * lse2r).sum() + (b * z2r).sum()).backward()
    torch.cuda.synchronize()
    assert _rel_err(lse2, lse2r) < 1e-2 and _rel_err(z2, z2r) < 2e-2
    assert _rel_err(f.grad, fr.grad) < 3e-2


@pytest.mark.parametrize("M", [1, 5, 16, 17, 32, 33, 64])
def test_skinny_tensor_core_gemm(cuda_device, M):
    """Swap-AB tcgen05 GEMM for a few rows: store / residual / SwiGLU against fp32, rows independent of M
    (M <= 16 runs the 16-row token tile, 17..32 the 32-row tile, 33..64 the 64-row tile; row 0 must
    match a 1-row call bitwise)."""
    ext = _ext()
    K, N = 4096, 1536
    x = (torch.randn(M, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device) * 0.02).to(torch.bfloat16)
    splits = int(ext.skinny_splits(N, K))
    ws = torch.empty(splits * N * 64, device=cuda_device)
    out = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    ext.skinny_gemm(x, w, 0, out, None, ws)
    ref = x.float() @ w.float().T
    res = torch.randn(M, N, device=cuda_device).to(torch.bfloat16)
    out_r = res.clone()
    ext.skinny_gemm(x, w, 1, out_r, out_r, ws)
    act = torch.empty(M, N // 2, device=cuda_device, dtype=torch.bfloat16)
    ext.skinny_gemm(x, w, 2, act, None, ws)
    one = torch.empty(1, N, device=cuda_device, dtype=torch.bfloat16)
    ext.skinny_gemm(x[:1].contiguous(), w, 0, one, None, ws)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert _rel_err(out, ref) < 1e-2
    assert _rel_err(out_r, res.float() + ref.to(torch.bfloat16).float()) < 1e-2
    g, u = ref.view(M, N // 256, 2, 128)[:, :, 0].reshape(M, -1), ref.view(M, N // 256, 2, 128)[:, :, 1].reshape(M, -1)
    assert _rel_err(act, torch.nn.functional.silu(g) * u) < 2e-2
    assert torch.equal(out[:1], one)


def test_skinny_qkv_allreduce_and_row_argmax(cuda_device):
    """Skinny QKV (RoPE + cache) against the GEMV QKV, the all-reduce epilogue on one rank, row argmax."""
    cfg = get_model_config("tiny128")
    ext = _ext()
    nq, nkv, K, cap, M = 4, 2, 512, 300, 5
    x = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn((nq + 2 * nkv) * 128, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    table = rope_table(cfg, 1024, cuda_device)
    pos = torch.tensor([123], device=cuda_device, dtype=torch.int32)
    ws = torch.empty(64 * 4096 * 16, device=cuda_device)
    outs = []
    for fn in ("gemv", "skinny"):
        kc = torch.zeros(nkv, cap, 128, device=cuda_device, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        q = torch.empty(M, nq * 128, device=cuda_device, dtype=torch.bfloat16)
        if fn == "gemv":
            ext.gemv_qkv(x, w, None, 1e-5, q, kc, vc, pos, table, nq, nkv)
        else:
            ext.skinny_qkv(x, w, q, kc, vc, pos, table, nq, nkv, ws)
        outs.append((q, kc, vc))
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    for a, b in zip(outs[0], outs[1]):
        assert _rel_err(b, a.float()) < 2e-2
    assert outs[1][1][:, 123:123 + M].abs().sum() > 0 and outs[1][1][:, 123 + M:].abs().sum() == 0
    # all-reduce epilogue, one rank: the partial rows land in the receive slot and the flag is released
    N = 1024
    w2 = (torch.randn(N, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    recv = torch.zeros(1, M, N, device=cuda_device)
    flags = torch.zeros(2, device=cuda_device, dtype=torch.int32)
    counter = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    ext.skinny_allreduce(x, w2, [recv.data_ptr()], [flags.data_ptr()], 0, 7, None, 0, counter, ws)
    torch.cuda.synchronize()
    assert _rel_err(recv[0], x.float() @ w2.float().T) < 1e-2
    assert int(flags[0]) == 7 and int(counter[0]) == 0
    # row argmax: first index on ties, as torch.argmax
    logits = torch.randn(M, 128256, device=cuda_device).to(torch.bfloat16)
    logits[2, 100] = logits[2, 5000] = 50.0
    tok = torch.empty(M, device=cuda_device, dtype=torch.int32)
    ext.row_argmax(logits, tok)
    torch.cuda.synchronize()
    assert tok.tolist() == logits.float().argmax(-1).tolist() and int(tok[2]) == 100


@pytest.mark.parametrize("M,N,K", [(1, 8192, 1024), (3, 4096, 2048), (8, 4096, 512)])
def test_gemv_allreduce_one_rank_matches_residual_gemv(cuda_device, M, N, K):
    """The decode all-reduce epilogue at one rank: each CTA's contiguous chunk
    of fp32 partials goes to the receive slot with vector stores, the flag is
    released, and the column-split reduce adds it to the residual; equal to
    the residual GEMV (same rounding order) twice in a row."""
    ext = _ext()
    g = torch.Generator(device="cpu").manual_seed(M * 1000 + N + K)
    x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(cuda_device, torch.bfloat16)
    res = torch.randn(M, N, generator=g).to(cuda_device, torch.bfloat16)
    recv = torch.zeros(1, M, N, device=cuda_device)
    flag = torch.zeros(4, device=cuda_device, dtype=torch.int32)
    counter = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    status = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    expect = torch.empty_like(res)
    ext.gemv_residual(x, w, None, 1e-5, expect, res)
    for epoch in (1, 2):
        out = res.clone()
        ext.gemv_allreduce(x, w, None, 1e-5, [recv.data_ptr()], [flag.data_ptr()], 0, epoch, None, 0, counter)
        ext.rs_reduce(recv, flag, epoch, int(2e9), status, out, out, None, None, 1e-5, None, 0)
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and int(flag[0].item()) == epoch
        torch.testing.assert_close(out.float(), expect.float(), rtol=0, atol=0)


@pytest.mark.parametrize("L,R,H,Hkv,T", [(1, 1, 32, 8, 16000), (3, 1, 8, 2, 777), (2, 4, 8, 8, 300)])
def test_page_token_scores_match_fp32_softmax(cuda_device, L, R, H, Hkv, T):
    """K11: mean over layers, query rows and heads of softmax(q K^T / sqrt(d)),
    per prompt token, against the fp32 einsum the reference uses."""
    ext = _ext()
    g = torch.Generator(device="cpu").manual_seed(L * 100 + T)
    cap = T + 37
    keys = [torch.randn(Hkv, cap, 128, generator=g).to(cuda_device, torch.bfloat16) for _ in range(L)]
    q = (torch.randn(L, R, H, 128, generator=g) * 1.5).to(cuda_device)
    got = ext.page_token_scores(q, keys, T, 128 ** -0.5)
    torch.cuda.synchronize()
    ref = torch.zeros(T, device=cuda_device)
    G = H // Hkv
    for l in range(L):
        k = keys[l][:, :T].float().repeat_interleave(G, dim=0)  # [H, T, D]
        logits = torch.einsum("rhd,htd->rht", q[l].float(), k) * 128 ** -0.5
        ref += logits.softmax(-1).mean(dim=(0, 1))
    ref /= L
    torch.testing.assert_close(got, ref, rtol=2e-3, atol=1e-6)
    assert abs(float(got.sum()) - 1.0) < 1e-3


# ------------------------------------------------ token-column GEMM (64 < M <= 512)
@pytest.mark.parametrize("M", [65, 130, 300, 512])
@pytest.mark.parametrize("acc,n_tt,splits", [(1, 0, 1), (2, 0, 3), (1, 3, 2), (0, 0, 0)])
def test_wide_gemm_store_and_residual(cuda_device, M, acc, n_tt, splits):
    """Weight tiles as the MMA's M, tokens as its N: every plan (weight tiles per unit, token
    tiles, K split) matches the fp32 reference, stored and with the residual epilogue."""
    ext = _ext()
    N, K = 1024, 1280
    if n_tt and -(-M // n_tt) > 256:
        pytest.skip("token tile wider than 256")
    g = torch.Generator(device="cpu").manual_seed(M * 3 + splits)
    x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.03).to(cuda_device, torch.bfloat16)
    res = torch.randn(M, N, generator=g).to(cuda_device, torch.bfloat16)
    out = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    assert ext.wide_residual(x, w, out, None, acc=acc, n_tt=n_tt, splits=splits) == 2
    out_r = res.clone()
    ext.wide_residual(x, w, out_r, out_r, acc=acc, n_tt=n_tt, splits=splits)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    y = x.float() @ w.float().T
    assert _rel_err(out, y) < 1e-2
    assert _rel_err(out_r, res.float() + y.to(torch.bfloat16).float()) < 1e-2


@pytest.mark.parametrize("M", [100, 300, 330])
def test_wide_swiglu_and_fused_norm(cuda_device, M):
    """Gate/up block pairs per unit with the SwiGLU epilogue; residual + RMSNorm through the
    split-K reduce is bit-identical to the norm kernel on the stored rows."""
    ext = _ext()
    K, F = 1024, 2048
    g = torch.Generator(device="cpu").manual_seed(M)
    x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    wg = (torch.randn(F, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    wu = (torch.randn(F, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    act = torch.empty(M, F, device=cuda_device, dtype=torch.bfloat16)
    assert ext.wide_swiglu(x, interleave_gate_up(wg, wu), act) == 1
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    gate = (x.float() @ wg.float().T).to(torch.bfloat16)
    up = (x.float() @ wu.float().T).to(torch.bfloat16)
    ref = torch.nn.functional.silu(gate.float()).to(torch.bfloat16).float() * up.float()
    assert _rel_err(act, ref) < 2e-2

    wd = (torch.randn(K, F, generator=g) * 0.02).to(cuda_device, torch.bfloat16)
    res = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, generator=g)).to(cuda_device, torch.bfloat16)
    h, normed = res.clone(), torch.empty(M, K, device=cuda_device, dtype=torch.bfloat16)
    ext.wide_residual(act, wd, h, h, norm_w=nw, eps=1e-5, norm_out=normed)
    ref_norm = torch.empty_like(normed)
    ext.rmsnorm(h, None, nw, 1e-5, ref_norm)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert torch.equal(normed, ref_norm)
    assert _rel_err(h, res.float() + (act.float() @ wd.float().T).to(torch.bfloat16).float()) < 1e-2


@pytest.mark.parametrize("M", [90, 300])
def test_wide_qkv_rope_scatter(cuda_device, M):
    """Token-column QKV: RoPE at per-row positions, Q rows out, K/V at per-row cache slots."""
    cfg = get_model_config("tiny128")
    nq, nkv, K, cap = 4, 2, 512, 600
    a = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn((nq + 2 * nkv) * 128, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    pos = torch.sort(torch.randperm(500)[:M]).values.to(torch.int32).to(cuda_device) + 7
    slot = torch.sort(torch.randperm(cap)[:M]).values.to(torch.int32).to(cuda_device)
    kc = torch.randn(nkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    vc = torch.randn(nkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    kc0 = kc.clone()
    q_out = torch.empty(M, nq * 128, device=cuda_device, dtype=torch.bfloat16)
    table = rope_table(cfg, 1024, cuda_device)
    assert _ext().wide_qkv(a, w, q_out, kc, vc, pos, slot, table, nq, nkv) == 2
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    q, k, v = _qkv_reference(a, w, cfg, pos, nq, nkv)
    assert _rel_err(q_out.reshape(M, nq, 128), q) < 1e-2
    sl = slot.long()
    assert _rel_err(kc[:, sl].transpose(0, 1), k) < 1e-2
    assert _rel_err(vc[:, sl].transpose(0, 1), v) < 1e-2
    untouched = torch.ones(cap, dtype=torch.bool, device=cuda_device)
    untouched[sl] = False
    assert torch.equal(kc[:, untouched], kc0[:, untouched])


@pytest.mark.parametrize("M,K", [(330, 1024), (300, 512)])
def test_wide_swiglu_stream_k_tail(cuda_device, M, K):
    """Units that do not fill whole rounds of the grid: the tail is cut into equal runs of
    k-blocks per CTA and the pieces of a unit are summed in piece order by the last one to
    arrive.  Matches the fp32 reference, repeats bit for bit, and leaves the arrival
    counters at zero (a second launch reads them)."""
    ext = _ext()
    F = 14336 if M == 330 else 10240
    plan = ext.wide_plan(M, 2 * F, K, 1)
    if ext.num_sms() == 148:
        assert plan["sk_tail"] > 0, plan
    g = torch.Generator(device="cpu").manual_seed(M + K)
    x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    wg = (torch.randn(F, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    wu = (torch.randn(F, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    wgu = interleave_gate_up(wg, wu)
    outs = []
    for _ in range(2):
        act = torch.empty(M, F, device=cuda_device, dtype=torch.bfloat16)
        ext.wide_swiglu(x, wgu, act)
        outs.append(act)
    ext.set_wide_stream_k(False)
    try:
        plain = torch.empty(M, F, device=cuda_device, dtype=torch.bfloat16)
        ext.wide_swiglu(x, wgu, plain)
    finally:
        ext.set_wide_stream_k(True)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    gate = (x.float() @ wg.float().T).to(torch.bfloat16)
    up = (x.float() @ wu.float().T).to(torch.bfloat16)
    ref = torch.nn.functional.silu(gate.float()).to(torch.bfloat16).float() * up.float()
    assert torch.equal(outs[0], outs[1])
    assert _rel_err(outs[0], ref) < 2e-2
    assert _rel_err(plain, ref) < 2e-2
