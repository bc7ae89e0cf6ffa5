"""The fms-shaped telescoping layer (telescope_cache_b200.fms_attention):
its forward and the gradients of every parameter and of the input against
torch autograd of a dense fp32 restatement of the reference's composition
(projections, short conv, merge weights, the dyadic tree of
reference.py:465-584, attention over exactly each query's visible set with
softcap / RoPE at summary positions / relative bias (reference.py:771-1071),
sink (reference.py:1082-1110), gate (reference.py:1187-1219), output
projection), on the same parameters.  The visible sets come from the CPU
oracle's schedule.  Decode through the layer equals the full forward.
Tolerance: fp32 normwise 1e-4; bf16 normwise 2e-2."""

import math

import pytest
import torch

from oracle import schedule as S
from telescope_cache_b200.fms_attention import MultiHeadAttention

pytestmark = pytest.mark.gpu


def _close(got, want, tol, what=""):
    got, want = got.detach().double().cpu(), want.detach().double().cpu()
    rel = ((got - want).norm() / max(want.norm().item(), 1e-30)).item()
    assert rel <= tol, f"{what}: normwise {rel:.3e} > {tol}"


def _visible(N, fmap, cache):
    """Per query: flat node index (level-major offsets), bin distance and
    summary position of each visible entry, padded to the widest row."""
    a = S.activation_times(fmap)
    L = len(a) - 1
    offs = S.level_offsets(N, L + 1)
    rows = [S.visible_entries(t, a, cache) for t in range(N)]
    M = max(len(r) for r in rows)
    idx = torch.zeros(N, M, dtype=torch.long)
    dist = torch.zeros(N, M, dtype=torch.long)
    ok = torch.zeros(N, M, dtype=torch.bool)
    for t, r in enumerate(rows):
        for m, (lv, j) in enumerate(r):
            idx[t, m] = offs[lv] + j
            dist[t, m] = len(r) - 1 - m
            ok[t, m] = True
    kpos = torch.cat([(torch.arange(N >> lv) + 1) * (1 << lv) - 1 for lv in range(L + 1)])
    return idx, dist, ok, kpos, L


def _rot(x, pos, cos, sin):
    c, s = cos[pos], sin[pos]
    h = x.shape[-1] // 2
    a, b = x[..., :h], x[..., h:]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def _dense(P, x, m: MultiHeadAttention):
    """The reference composition in fp32 torch ops over the leaves P."""
    B, N, _ = x.shape
    H, Hkv, Dk, Dv = m.nheads, m.kvheads, m.emb_kq_per_head, m.emb_v_per_head
    E = H // Hkv
    q, k, v = torch.split(x @ P["in_proj.weight"].t(), m._split, dim=-1)
    if m.use_kv_short_conv:
        def conv(z, w):
            K = w.shape[1]
            zp = torch.nn.functional.pad(z, (0, 0, K - 1, 0))
            return z + sum(w[:, j] * zp[:, j:j + N] for j in range(K))
        k, v = conv(k, P["k_sconv.weight"]), conv(v, P["v_sconv.weight"])
    q, k, v = q.reshape(B, N, H, Dk), k.reshape(B, N, Hkv, Dk), v.reshape(B, N, Hkv, Dv)
    if m.weight_mode == "linear":
        w = x @ P["w.weight"].t()
    else:
        s = (q.reshape(B, N, Hkv, E, Dk) * k.unsqueeze(3)).sum(-1) / math.sqrt(Dk)
        w = torch.logsumexp(s, dim=3)
    idx, dist, ok, kpos, L = _visible(N, m.fmap, m.cache_size)
    ks, vs, ws = [k], [v], [w]
    for _ in range(L):
        u = ks[-1].shape[1] // 2
        wp = ws[-1][:, :2 * u].reshape(B, u, 2, Hkv)
        al = torch.softmax(wp, dim=2).unsqueeze(-1)
        ks.append((al * ks[-1][:, :2 * u].reshape(B, u, 2, Hkv, Dk)).sum(2))
        vs.append((al * vs[-1][:, :2 * u].reshape(B, u, 2, Hkv, Dv)).sum(2))
        ws.append(torch.logsumexp(wp, dim=2))
    K_all, V_all = torch.cat(ks, dim=1), torch.cat(vs, dim=1)
    dev = x.device
    idx, dist, ok, kpos = idx.to(dev), dist.to(dev), ok.to(dev), kpos.to(dev)
    qq = q
    if m.position_mode == "rope":
        cos, sin = m._rope_tables(N, dev)
        qq = _rot(q, torch.arange(N, device=dev)[None, :, None], cos, sin)
        K_all = _rot(K_all, kpos[None, :, None], cos, sin)
    Kg = K_all[:, idx].repeat_interleave(E, dim=3)  # [B, N, M, H, Dk]
    Vg = V_all[:, idx].repeat_interleave(E, dim=3)
    X = torch.einsum("bthd,btmhd->bthm", qq, Kg) / math.sqrt(Dk)
    if m.position_mode == "relative":
        st = (x @ P["relative_weight"].t()).reshape(B, N, H, -1)
        rel = st @ P["relative_proj"]  # [B, N, H, bins]
        X = X + torch.gather(rel, 3, dist[None, :, None, :].expand(B, N, H, -1))
    Sx = m.softcap * torch.tanh(X / m.softcap) if m.softcap is not None else X
    Sx = Sx.masked_fill(~ok[None, :, None, :], float("-inf"))
    lse = torch.logsumexp(Sx, dim=-1)
    out = torch.einsum("bthm,btmhd->bthd", torch.exp(Sx - lse.unsqueeze(-1)), Vg)
    if m.use_sinks:
        out = out * torch.sigmoid(lse - P["sinks"]).unsqueeze(-1)
    if m.use_gate:
        out = torch.nn.functional.silu(x @ P["gate_proj.weight"].t()).reshape(B, N, H, Dv) * out
    return out.reshape(B, N, H * Dv) @ P["dense.weight"].t()


CASES = [
    # fp32 (SIMT kernels), every feature, three position modes
    dict(dtype=torch.float32, B=2, N=96, emb=32, H=8, Hkv=4, D=16, fmap={1: 4, 2: 6, 3: 8}, cache=12,
         weight_mode="qk", conv=True, sinks=True, gate=True, pos="none", tol=1e-4),
    dict(dtype=torch.float32, B=2, N=96, emb=32, H=8, Hkv=4, D=16, fmap={1: 4, 2: 6, 3: 8}, cache=12,
         weight_mode="linear", conv=True, sinks=True, gate=True, pos="rope", tol=1e-4),
    dict(dtype=torch.float32, B=1, N=96, emb=32, H=4, Hkv=2, D=16, fmap={1: 4, 2: 6, 3: 8}, cache=12,
         weight_mode="qk", conv=False, sinks=False, gate=False, pos="relative", tol=1e-4),
    # bf16 head dim 128 (tensor-core kernels)
    dict(dtype=torch.bfloat16, B=1, N=512, emb=256, H=4, Hkv=2, D=128, fmap={1: 64, 2: 128, 3: 192},
         cache=256, weight_mode="qk", conv=True, sinks=True, gate=True, pos="rope", tol=2e-2),
    dict(dtype=torch.bfloat16, B=1, N=512, emb=256, H=2, Hkv=1, D=128, fmap={1: 64, 2: 128, 3: 192},
         cache=256, weight_mode="linear", conv=False, sinks=True, gate=False, pos="relative", tol=2e-2),
]


def _layer(c, seed):
    torch.manual_seed(seed)
    m = MultiHeadAttention(c["emb"], c["D"], c["D"], c["H"], c["Hkv"], fmap=c["fmap"], cache_size=c["cache"],
                           weight_mode=c["weight_mode"], use_kv_short_conv=c["conv"], use_sinks=c["sinks"],
                           use_gate=c["gate"], position_mode=c["pos"])
    with torch.no_grad():
        # non-trivial conv, sinks and projections (fms initialises them near zero)
        for name, p in m.named_parameters():
            if name.endswith("sconv.weight") or name == "sinks":
                p.copy_(torch.randn_like(p) * 0.3)
            else:
                p.copy_(torch.randn_like(p) / math.sqrt(p.shape[-1]))
    return m.cuda().to(c["dtype"])


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_layer_forward_and_gradients_match_dense_restatement(ci):
    c = CASES[ci]
    torch.cuda.set_device(0)
    m = _layer(c, 100 + ci)
    g = torch.Generator(device="cuda")
    g.manual_seed(200 + ci)
    x = torch.randn(c["B"], c["N"], c["emb"], generator=g, device="cuda").to(c["dtype"])
    dy = torch.randn(c["B"], c["N"], c["emb"], generator=g, device="cuda").to(c["dtype"])
    x1 = x.clone().requires_grad_(True)
    y = m(x1)
    assert y.dtype == c["dtype"] and y.shape == x.shape
    names = [n for n, _ in m.named_parameters()]
    grads = torch.autograd.grad(y, [x1] + [p for _, p in m.named_parameters()], dy)
    P = {n: p.detach().float().clone().requires_grad_(True) for n, p in m.named_parameters()}
    x2 = x.float().clone().requires_grad_(True)
    y2 = _dense(P, x2, m)
    want = torch.autograd.grad(y2, [x2] + [P[n] for n in names], dy.float())
    _close(y, y2, c["tol"], "out")
    for n, a, b_ in zip(["x"] + names, grads, want):
        assert a.dtype == (x.dtype if n == "x" else dict(m.named_parameters())[n].dtype)
        _close(a, b_, c["tol"], f"d{n}")


@pytest.mark.parametrize("ci", [0, 1, 2, 3, 4])
def test_layer_decode_equals_forward(ci):
    c = CASES[ci]
    torch.cuda.set_device(0)
    m = _layer(c, 300 + ci)
    g = torch.Generator(device="cuda")
    g.manual_seed(400 + ci)
    x = torch.randn(c["B"], c["N"], c["emb"], generator=g, device="cuda").to(c["dtype"])
    n0, steps = c["N"] - 5, 5
    with torch.no_grad():
        full = m(x)
        y0, state = m(x[:, :n0], use_cache=True)
        _close(y0, full[:, :n0], c["tol"], "prefill")
        outs = [m.decode(x[:, t:t + 1], state) for t in range(n0, n0 + steps)]
    assert state.t == c["N"]
    _close(torch.cat(outs, dim=1), full[:, n0:], c["tol"], "decode")


def test_layer_rejects_what_it_does_not_implement():
    with pytest.raises(NotImplementedError):
        MultiHeadAttention(32, 16, 16, 4, 2, p_dropout=0.1)
    with pytest.raises(NotImplementedError):
        MultiHeadAttention(32, 16, 16, 4, 2, weight_mode=None)
    with pytest.raises(NotImplementedError):
        MultiHeadAttention(32, 16, 16, 4, 2, position_encoder=object())
    m = MultiHeadAttention(32, 16, 16, 4, 2, fmap={1: 4, 2: 6, 3: 8}, cache_size=12).cuda()
    x = torch.randn(1, 16, 32, device="cuda")
    with pytest.raises(NotImplementedError):
        m(x, mask=torch.ones(16, 16, dtype=torch.bool, device="cuda"))
    with pytest.raises(NotImplementedError):
        m(x, is_self=False)
