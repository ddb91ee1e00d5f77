"""The tnn_* primitive op surface (lazy graph + autograd) through the C ABI.

Forward ops are checked against numpy float64 with ggml's shape convention
(a tensor with ne = [ne0, ne1, ne2] is the row-major array of shape
(ne2, ne1, ne0)); matrix products run on the split-bf16 tensor-core GEMM
(2e-5 relative), everything else in f32 (1e-5). The explicit backward
primitives are checked against their formulas, including the reference's
recorded RMSNorm-back known answer (tinynn/rms_norm_back_probe.c: [0.0008, 0,
0, 0]). Autograd is checked on a one-layer Llama block built op by op the
way toy's graph builders do (embedding, RMSNorm, grouped-query attention with
RoPE, causal mask and softmax, SwiGLU FFN, tied LM head, cross-entropy)
against torch float64 autograd: loss 1e-4 relative, every parameter gradient
and the AdamW-updated parameters 1e-3 relative L2.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (nb if nb > 0 else 1.0)


class Graph:
    """Thin helper over the C calls (one session per graph)."""

    def __init__(self):
        from toy_b200._lib import lib
        self.L = lib()
        self.s = self.L.tnn_session_new(1)
        assert self.s

    def close(self):
        self.L.tnn_session_free(self.s)

    def f32(self, arr, persistent=True):
        arr = np.ascontiguousarray(arr, np.float64)
        ne = list(arr.shape[::-1])
        L = self.L
        if not persistent:
            assert arr.ndim <= 2
            t = L.tnn_input_2d_f32(self.s, ne[1] if arr.ndim == 2 else 1, ne[0])
        elif arr.ndim == 1:
            t = L.tnn_input_1d_f32_persistent(self.s, ne[0])
        elif arr.ndim == 2:
            t = L.tnn_input_2d_f32_persistent(self.s, ne[1], ne[0])
        elif arr.ndim == 3:
            t = L.tnn_input_3d_f32_persistent(self.s, ne[0], ne[1], ne[2])
        else:
            t = L.tnn_input_4d_f32_persistent(self.s, ne[0], ne[1], ne[2], ne[3])
        assert t
        if persistent:
            self.put(t, arr)
        return t

    def put(self, t, arr):
        arr = np.ascontiguousarray(arr, np.float64).reshape(-1)
        assert self.L.tnn_upload_from_float_array(self.s, t, arr.ctypes.data_as(C.POINTER(C.c_double)),
                                                  arr.size) == 0

    def i32(self, arr):
        arr = np.ascontiguousarray(arr, np.int64)
        t = self.L.tnn_input_1d_i32_ctx(self.s, arr.size)
        assert t and self.L.tnn_upload_from_int_array(self.s, t, arr.ctypes.data_as(C.POINTER(C.c_long)),
                                                      arr.size) == 0
        return t

    def get(self, t):
        L = self.L
        ne = [L.tnn_tensor_ne0(t), L.tnn_tensor_ne1(t), L.tnn_tensor_ne2(t), L.tnn_tensor_ne3(t)]
        out = np.empty(int(np.prod(ne)), np.float64)
        assert L.tnn_download_to_f64_array(self.s, t, out.ctypes.data_as(C.POINTER(C.c_double)), out.size) == 0
        shape = [n for n in ne[::-1]]
        while len(shape) > 1 and shape[0] == 1:
            shape = shape[1:]
        return out.reshape(shape)

    def run(self, outputs):
        for t in outputs:
            assert t
            self.L.tnn_set_output(t)
        assert self.L.tnn_realize(self.s, outputs[-1]) == 0
        assert self.L.tnn_compute(self.s) == 0
        return [self.get(t) for t in outputs]


def rope_ref(x, pos, n_dims, base, fscale=1.0, ff=None, attn=1.0, inverse=False):
    """NEOX RoPE on x of shape (T, H, dh) with ggml's f32 theta recurrence."""
    x = np.asarray(x, np.float64)
    out = x.copy()
    half = n_dims // 2
    ts = np.float32(np.float32(base) ** np.float32(-2.0 / n_dims))
    for t in range(x.shape[0]):
        theta = np.float32(pos[t])
        for i in range(half):
            f = np.float32(1.0 if ff is None else ff[i])
            th = np.float32(np.float32(fscale) * np.float32(theta / f))
            c = np.float64(np.float32(np.cos(np.float32(th))) * np.float32(attn))
            s = np.float64(np.float32(np.sin(np.float32(th))) * np.float32(attn)) * (-1.0 if inverse else 1.0)
            x0, x1 = x[t, :, i], x[t, :, i + half]
            out[t, :, i] = x0 * c - x1 * s
            out[t, :, i + half] = x0 * s + x1 * c
            theta = np.float32(theta * ts)
    return out


def softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def test_forward_ops(cuda):
    rng = np.random.default_rng(0)
    g = Graph()
    L, s = g.L, g.s
    A = rng.standard_normal((96, 64)); Bm = rng.standard_normal((40, 64))
    a, b = g.f32(A), g.f32(Bm)
    mm = L.tnn_matmul(s, a, b)                                     # (40, 96) = B A^T
    A3 = rng.standard_normal((2, 48, 64)); B3 = rng.standard_normal((6, 40, 64))
    mm3 = L.tnn_matmul(s, g.f32(A3), g.f32(B3))                   # GQA broadcast: batch z reads z // 3
    OA = rng.standard_normal((50, 24)); OB = rng.standard_normal((50, 32))
    op = L.tnn_out_prod(s, g.f32(OA), g.f32(OB))                   # (32, 24) = OB^T OA
    X = rng.standard_normal((5, 7, 16)); bias = rng.standard_normal(16)
    xt = g.f32(X)
    ad = L.tnn_add(s, xt, g.f32(bias))
    mu = L.tnn_mul(s, xt, g.f32(X * 0.5))
    sc = L.tnn_scale(s, xt, -1.5)
    si = L.tnn_silu(s, xt)
    Up = rng.standard_normal((5, 7, 16))
    sw = L.tnn_swiglu_split(s, xt, g.f32(Up))
    gam = rng.standard_normal(16)
    rn = L.tnn_rms_norm(s, xt, g.f32(gam.reshape(1, 16)), 1e-5)
    tr = L.tnn_transpose(s, g.f32(A))
    pm = L.tnn_permute(s, xt, 1, 0, 2, 3)
    cc = L.tnn_concat(s, xt, g.f32(Up), 1)
    E = rng.standard_normal((30, 16)); ids = np.array([3, 0, 29, 3, 7])
    gr = L.tnn_get_rows(s, g.f32(E), g.i32(ids))
    sr = L.tnn_sum_rows(s, xt)
    su = L.tnn_sum(s, xt)
    v2 = L.tnn_view_2d(s, g.f32(A), 8, 10, 64 * 4 * 8, 16 * 4)     # rows 0, 8, .., 72; columns 16..23
    Z = rng.standard_normal((12, 40)); Y = softmax(rng.standard_normal((12, 40)) * 3)
    ce = L.tnn_cross_entropy_loss(s, g.f32(Z), g.f32(Y))
    outs = g.run([mm, mm3, op, ad, mu, sc, si, sw, rn, tr, pm, cc, gr, sr, su, v2, ce])
    (r_mm, r_mm3, r_op, r_ad, r_mu, r_sc, r_si, r_sw, r_rn, r_tr, r_pm, r_cc, r_gr, r_sr, r_su, r_v2, r_ce) = outs
    assert rel(r_mm, Bm @ A.T) < 2e-5
    ref3 = np.stack([B3[z] @ A3[z // 3].T for z in range(6)])
    assert rel(r_mm3, ref3) < 2e-5
    assert rel(r_op, OB.T @ OA) < 2e-5
    assert rel(r_ad, X + bias) < 1e-6
    assert rel(r_mu, X * X * 0.5) < 1e-6
    assert rel(r_sc, -1.5 * X) < 1e-6
    assert rel(r_si, X / (1 + np.exp(-X))) < 1e-5
    assert rel(r_sw, X / (1 + np.exp(-X)) * Up) < 1e-5
    assert rel(r_rn, X / np.sqrt((X * X).mean(-1, keepdims=True) + 1e-5) * gam) < 1e-5
    f32 = lambda x: np.asarray(x, np.float32).astype(np.float64)   # copies are exact on the f32 inputs
    assert rel(r_tr, f32(A).T) == 0
    assert rel(r_pm, f32(X).transpose(0, 2, 1)) == 0
    assert rel(r_cc, f32(np.concatenate([X, Up], axis=1))) == 0
    assert rel(r_gr, f32(E[ids])) == 0
    assert rel(r_sr.reshape(5, 7), X.sum(-1)) < 1e-6
    assert abs(float(r_su.reshape(-1)[0]) - X.sum()) < 1e-4 * np.abs(X).sum()
    assert rel(r_v2, f32(A[0:80:8, 16:24])) == 0
    ref_ce = -(Y * np.log(softmax(Z))).sum(-1).mean()
    assert abs(float(r_ce.reshape(-1)[0]) - ref_ce) < 1e-5 * abs(ref_ce)
    g.close()


def test_attention_ops(cuda):
    rng = np.random.default_rng(1)
    g = Graph()
    L, s = g.L, g.s
    T, H, dh = 6, 3, 16
    X = rng.standard_normal((T, H, dh))
    pos = np.arange(T) + 2
    ffac = np.array([1.0, 1.0, 2.0, 4.0, 1.0, 8.0, 1.0, 2.0])
    ff = L.tnn_rope_freq_factors_alloc(s, dh)
    g.put(ff, ffac)
    pt = g.i32(pos)
    xt = g.f32(X)
    ro = L.tnn_rope_ext(s, xt, pt, dh, 1e4, 1.0, 0.0, 1.0, 32.0, 1.0, ff)
    rb = L.tnn_rope_ext_back(s, xt, pt, dh, 1e4, 1.0, 0.0, 1.0, 32.0, 1.0, ff)
    S = rng.standard_normal((H, T, T))
    mask = np.where(np.arange(T)[None, :] > np.arange(T)[:, None], -np.inf, 0.0)
    st = g.f32(S)
    sm = L.tnn_softmax(s, st)
    mk = g.f32(np.nan_to_num(mask, neginf=-1e30))
    se = L.tnn_soft_max_ext(s, st, mk, 0.25, 0.0)
    dm = L.tnn_diag_mask_inf(s, st, 1)
    r_ro, r_rb, r_sm, r_se, r_dm = g.run([ro, rb, sm, se, dm])
    assert rel(r_ro, rope_ref(X, pos, dh, 1e4, ff=ffac)) < 1e-5
    assert rel(r_rb, rope_ref(X, pos, dh, 1e4, ff=ffac, inverse=True)) < 1e-5
    assert rel(r_sm, softmax(S)) < 1e-5
    assert rel(r_se, softmax(0.25 * S + np.nan_to_num(mask, neginf=-1e30))) < 1e-5
    ref_dm = S.copy()
    ref_dm[:, np.arange(T)[:, None] + 1 < np.arange(T)[None, :]] = -np.inf
    assert np.array_equal(np.isinf(r_dm), np.isinf(ref_dm))
    assert rel(np.where(np.isinf(ref_dm), 0, r_dm), np.where(np.isinf(ref_dm), 0, np.float32(ref_dm))) == 0
    g.close()


def test_q8_0_matmul(cuda):
    from oracle import oracle as O
    rng = np.random.default_rng(2)
    g = Graph()
    L, s = g.L, g.s
    W = 0.02 * rng.standard_normal((80, 128))
    Xb = rng.standard_normal((33, 128))
    wq = L.tnn_input_2d_persistent_typed(s, 80, 128, 8)
    blocks = O.q8_0_quantize(W.astype(np.float32))
    assert L.tnn_upload_q8_0_blocks(s, wq, blocks.ctypes.data, blocks.nbytes) == 0
    deq = O.q8_0_dequantize(blocks, 128)
    head = L.tnn_view_2d(s, wq, 128, 16, L.tnn_row_size(8, 128), 32 * L.tnn_row_size(8, 128))   # rows 32..47
    y = L.tnn_matmul(s, wq, g.f32(Xb))
    yh = L.tnn_matmul(s, head, g.f32(Xb))
    r_y, r_yh = g.run([y, yh])
    assert rel(r_y, Xb @ deq.T) < 2e-5
    assert rel(r_yh, Xb @ deq[32:48].T) < 2e-5
    assert rel(g.get(wq), deq) == 0   # download dequantises the blocks
    g.close()


def test_backward_primitives(cuda):
    rng = np.random.default_rng(3)
    g = Graph()
    L, s = g.L, g.s
    # tinynn/rms_norm_back_probe.c: x = dz = [1, 0, 0, 0], eps 1e-4 -> [0.0008, 0, 0, 0]
    x1 = g.f32(np.array([[1.0, 0, 0, 0]]))
    rb = L.tnn_rms_norm_back(s, x1, g.f32(np.array([[1.0, 0, 0, 0]])), 1e-4)
    X = rng.standard_normal((4, 24)); DY = rng.standard_normal((4, 24))
    xt, dyt = g.f32(X), g.f32(DY)
    rb2 = L.tnn_rms_norm_back(s, xt, dyt, 1e-5)
    sb = L.tnn_silu_back(s, xt, dyt)
    Ysm = softmax(X)
    smb = L.tnn_softmax_back(s, g.f32(Ysm), dyt)
    ids = np.array([2, 5, 2, 0])
    grb = L.tnn_get_rows_back(s, dyt, g.i32(ids), g.f32(np.zeros((7, 24))))
    r_rb, r_rb2, r_sb, r_smb, r_grb = g.run([rb, rb2, sb, smb, grb])
    assert np.allclose(r_rb.reshape(-1), [0.0008, 0, 0, 0], atol=1e-6)   # exact: 7.9952e-4
    n = X.shape[1]
    ss = (X * X).sum(-1, keepdims=True)
    ref = (DY - X * (X * DY).sum(-1, keepdims=True) / (ss + n * 1e-5)) / np.sqrt(ss / n + 1e-5)
    assert rel(r_rb2, ref) < 1e-5
    sg = 1 / (1 + np.exp(-X))
    assert rel(r_sb, DY * sg * (1 + X * (1 - sg))) < 1e-5
    assert rel(r_smb, Ysm * (DY - (Ysm * DY).sum(-1, keepdims=True))) < 1e-5
    ref_g = np.zeros((7, 24))
    for i, r in enumerate(ids):
        ref_g[r] += DY[i]
    assert rel(r_grb, ref_g) < 1e-6
    g.close()


# ------------------------------------------------------------------ autograd on a Llama block
CFG = dict(T=32, d=64, H=4, KV=2, dh=16, ff=128, V=96, eps=1e-5, base=1e4)


def block_params(rng):
    c = CFG
    p = {
        "E": 0.1 * rng.standard_normal((c["V"], c["d"])),
        "g1": 1 + 0.1 * rng.standard_normal(c["d"]),
        "Wq": rng.standard_normal((c["H"] * c["dh"], c["d"])) / 8,
        "Wk": rng.standard_normal((c["KV"] * c["dh"], c["d"])) / 8,
        "Wv": rng.standard_normal((c["KV"] * c["dh"], c["d"])) / 8,
        "Wo": rng.standard_normal((c["d"], c["H"] * c["dh"])) / 8,
        "g2": 1 + 0.1 * rng.standard_normal(c["d"]),
        "Wg": rng.standard_normal((c["ff"], c["d"])) / 8,
        "Wu": rng.standard_normal((c["ff"], c["d"])) / 8,
        "Wd": rng.standard_normal((c["d"], c["ff"])) / 11,
        "gf": 1 + 0.1 * rng.standard_normal(c["d"]),
    }
    ids = rng.integers(0, c["V"], c["T"])
    labels = np.zeros((c["T"], c["V"]))
    labels[np.arange(c["T"]), np.roll(ids, -1)] = 1.0
    return p, ids, labels


def torch_block(p, ids, labels):
    import torch
    c = CFG
    T, d, H, KV, dh = c["T"], c["d"], c["H"], c["KV"], c["dh"]
    P = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True) for k, v in p.items()}

    def rms(x, gm):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + c["eps"]) * gm

    def rope(x):   # x (T, heads, dh), NEOX with the f32 recurrence
        half = dh // 2
        ts = np.float32(np.float32(c["base"]) ** np.float32(-2.0 / dh))
        cos = np.zeros((T, half)); sin = np.zeros((T, half))
        for t in range(T):
            th = np.float32(t)
            for i in range(half):
                cos[t, i] = np.float32(np.cos(th)); sin[t, i] = np.float32(np.sin(th))
                th = np.float32(th * ts)
        cs, sn = torch.tensor(cos)[:, None, :], torch.tensor(sin)[:, None, :]
        x0, x1 = x[..., :half], x[..., half:]
        return torch.cat([x0 * cs - x1 * sn, x0 * sn + x1 * cs], -1)

    x0 = P["E"][torch.tensor(ids)]
    h = rms(x0, P["g1"])
    q = rope((h @ P["Wq"].T).reshape(T, H, dh))
    k = rope((h @ P["Wk"].T).reshape(T, KV, dh))
    v = (h @ P["Wv"].T).reshape(T, KV, dh)
    G = H // KV
    o = []
    for hh in range(H):
        sc = q[:, hh] @ k[:, hh // G].T / np.sqrt(dh)
        sc = sc.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
        o.append(torch.softmax(sc, -1) @ v[:, hh // G])
    o = torch.stack(o, 1).reshape(T, H * dh)
    x1 = x0 + o @ P["Wo"].T
    h2 = rms(x1, P["g2"])
    a = torch.nn.functional.silu(h2 @ P["Wg"].T) * (h2 @ P["Wu"].T)
    x2 = x1 + a @ P["Wd"].T
    logits = rms(x2, P["gf"]) @ P["E"].T
    loss = -(torch.tensor(labels) * torch.log_softmax(logits, -1)).sum(-1).mean()
    loss.backward()
    return loss.item(), {k2: t.grad.numpy() for k2, t in P.items()}


def build_block(g, p, ids, labels):
    """The block op by op, ggml style."""
    L, s = g.L, g.s
    c = CFG
    T, d, H, KV, dh = c["T"], c["d"], c["H"], c["KV"], c["dh"]
    P = {}
    for k, v in p.items():
        P[k] = g.f32(v if v.ndim == 2 else v.reshape(1, -1))
        L.tnn_set_param(P[k])
    idt = g.i32(ids)
    pos = g.i32(np.arange(T))
    lab = g.f32(labels)
    x0 = L.tnn_get_rows(s, P["E"], idt)                                    # [d, T]
    h = L.tnn_rms_norm(s, x0, P["g1"], c["eps"])
    def heads(W, n):   # [n*dh, T] -> [dh, n, T], roped
        y = L.tnn_reshape_3d(s, L.tnn_matmul(s, W, h), dh, n, T)
        return y
    q = L.tnn_rope_ext(s, heads(P["Wq"], H), pos, dh, c["base"], 1.0, 0.0, 1.0, 32.0, 1.0, None)
    k = L.tnn_rope_ext(s, heads(P["Wk"], KV), pos, dh, c["base"], 1.0, 0.0, 1.0, 32.0, 1.0, None)
    v = heads(P["Wv"], KV)
    qh = L.tnn_permute(s, q, 0, 2, 1, 3)                                  # [dh, T, H]
    kh = L.tnn_permute(s, k, 0, 2, 1, 3)                                  # [dh, T, KV]
    vt = L.tnn_permute(s, v, 1, 2, 0, 3)                                  # [T, dh, KV]
    kq = L.tnn_matmul(s, kh, qh)                                          # [T_k, T_q, H]
    kq = L.tnn_scale(s, kq, 1.0 / np.sqrt(dh))
    kq = L.tnn_diag_mask_inf(s, kq, 0)
    pr = L.tnn_softmax(s, kq)
    o = L.tnn_matmul(s, vt, pr)                                           # [dh, T_q, H]
    o = L.tnn_permute(s, o, 0, 2, 1, 3)                                   # [dh, H, T]
    o = L.tnn_reshape_2d(s, o, H * dh, T)
    x1 = L.tnn_add(s, x0, L.tnn_matmul(s, P["Wo"], o))
    h2 = L.tnn_rms_norm(s, x1, P["g2"], c["eps"])
    a = L.tnn_swiglu_split(s, L.tnn_matmul(s, P["Wg"], h2), L.tnn_matmul(s, P["Wu"], h2))
    x2 = L.tnn_add(s, x1, L.tnn_matmul(s, P["Wd"], a))
    logits = L.tnn_matmul(s, P["E"], L.tnn_rms_norm(s, x2, P["gf"], c["eps"]))
    loss = L.tnn_cross_entropy_loss(s, logits, lab)
    assert loss
    return P, loss


def test_autograd_llama_block(cuda):
    rng = np.random.default_rng(4)
    p, ids, labels = block_params(rng)
    ref_loss, ref_grads = torch_block(p, ids, labels)
    g = Graph()
    L, s = g.L, g.s
    P, loss = build_block(g, p, ids, labels)
    L.tnn_set_loss(loss)
    assert L.tnn_build_forward_only(s, loss) == 0
    assert L.tnn_build_backward(s) == 0
    grads = {k: L.tnn_tensor_grad(s, t) for k, t in P.items()}
    assert all(grads.values())
    assert L.tnn_realize_backward(s) == 0
    assert L.tnn_graph_reset(s) == 0
    assert L.tnn_compute_backward(s) == 0
    got = float(g.get(loss).reshape(-1)[0])
    assert abs(got - ref_loss) < 1e-4 * abs(ref_loss), (got, ref_loss)
    for k, t in grads.items():
        r = rel(g.get(t).reshape(ref_grads[k].shape), ref_grads[k])
        assert r < 1e-3, (k, r)
    # the backward program holds the node types ggml's autograd emits
    names = {L.tnn_tensor_op_name(L.tnn_graph_node(s, i)).decode() for i in range(L.tnn_graph_n_nodes(s))}
    for op in ("OUT_PROD", "RMS_NORM_BACK", "ROPE_BACK", "SOFT_MAX_BACK", "SILU_BACK", "CROSS_ENTROPY_LOSS_BACK",
               "GET_ROWS_BACK"):
        assert op in names, op
    g.close()


def test_opt_step_adamw_graph(cuda):
    rng = np.random.default_rng(5)
    p, ids, labels = block_params(rng)
    g = Graph()
    L, s = g.L, g.s
    P, loss = build_block(g, p, ids, labels)
    L.tnn_set_loss(loss)
    assert L.tnn_build_forward_only(s, loss) == 0 and L.tnn_build_backward(s) == 0
    hp = L.tnn_input_1d_f32_persistent(s, 7)
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    moments = {}
    for k, t in P.items():
        n = int(np.prod(p[k].shape))
        m, v = L.tnn_input_1d_f32_persistent(s, n), L.tnn_input_1d_f32_persistent(s, n)
        moments[k] = (m, v)
        step = L.tnn_opt_step_adamw(s, t, L.tnn_tensor_grad(s, t), m, v, hp)
        assert step and L.tnn_extend_backward_graph(s, step) == 0
    assert L.tnn_realize_backward(s) == 0
    ref = {k: v.copy() for k, v in p.items()}
    mref = {k: np.zeros_like(v) for k, v in p.items()}
    vref = {k: np.zeros_like(v) for k, v in p.items()}
    for it in (1, 2):
        g.put(hp, np.array([lr, b1, b2, eps, wd, 1 / (1 - b1 ** it), 1 / (1 - b2 ** it)]))
        assert (L.tnn_graph_reset(s) if it == 1 else L.tnn_graph_reset_grads_only(s)) == 0
        _, rg = torch_block(ref, ids, labels)
        assert L.tnn_compute_backward(s) == 0
        for k in ref:   # tinynn_ggml.h:457-465
            gk = rg[k]
            mref[k] = mref[k] * b1 + gk * (1 - b1)
            vref[k] = vref[k] * b2 + gk * gk * (1 - b2)
            ref[k] = ref[k] * (1 - lr * wd) - lr * (mref[k] / (1 - b1 ** it)) / (np.sqrt(vref[k] / (1 - b2 ** it)) + eps)
    for k, t in P.items():
        r = rel(g.get(t).reshape(ref[k].shape), ref[k])
        assert r < 1e-3, (k, r)
    g.close()


def test_cast_sgd_and_flash_attn_ext(cuda):
    from oracle import oracle as O
    rng = np.random.default_rng(6)
    g = Graph()
    L, s = g.L, g.s
    W = 0.05 * rng.standard_normal((6, 64))
    wq = L.tnn_input_2d_persistent_typed(s, 6, 64, 8)
    blocks = O.q8_0_quantize(W.astype(np.float32))
    assert L.tnn_upload_q8_0_blocks(s, wq, blocks.ctypes.data, blocks.nbytes) == 0
    deq = L.tnn_cast(s, wq, 0)                     # Q8_0 -> F32 (ggml_cast = CPY)
    X = rng.standard_normal((3, 8))
    cp = L.tnn_cast(s, g.f32(X), 0)
    assert not L.tnn_cast(s, wq, 30)               # bf16 target: not supported
    P0, G0 = rng.standard_normal(20), rng.standard_normal(20)
    p, gr = g.f32(P0), g.f32(G0)
    sgd = L.tnn_opt_step_sgd(s, p, gr, g.f32(np.array([0.1, 0.01])))
    # attention: B = 2, H = 4 query heads over KV = 2, dh = 16, causal mask
    B, Tq, Tk, H, KV, dh = 2, 5, 5, 4, 2, 16
    Q = rng.standard_normal((B, H, Tq, dh)); K = rng.standard_normal((B, KV, Tk, dh)); V = rng.standard_normal((B, KV, Tk, dh))
    mask = np.where(np.arange(Tk)[None, :] > np.arange(Tq)[:, None], -1e30, 0.0)
    fa = L.tnn_flash_attn_ext(s, g.f32(Q), g.f32(K), g.f32(V), g.f32(mask), 0.25, 0.0, 0.0)
    assert not L.tnn_flash_attn_ext(s, g.f32(Q), g.f32(K), g.f32(V), None, 0.25, 0.0, 30.0)   # softcap
    r_deq, r_cp, r_sgd, r_fa = g.run([deq, cp, sgd, fa])
    assert np.array_equal(r_deq.reshape(6, 64), O.q8_0_dequantize(blocks, 64).astype(np.float64))
    assert rel(r_cp, np.float32(X)) == 0
    ref = np.float32(P0) * (1 - 0.1 * 0.01) - 0.1 * np.float32(G0)
    assert rel(r_sgd.reshape(-1), ref) < 1e-6
    ref_o = np.zeros((B, Tq, H, dh))
    for b in range(B):
        for h in range(H):
            sc = 0.25 * Q[b, h] @ K[b, h // 2].T + mask
            ref_o[b, :, h] = softmax(sc) @ V[b, h // 2]
    assert rel(r_fa.reshape(B, Tq, H, dh), ref_o) < 2e-5
    g.close()


def test_scratch_mmap_and_transposed_upload(cuda):
    from oracle import oracle as O
    rng = np.random.default_rng(7)
    g = Graph()
    L, s = g.L, g.s
    # weights from an attached host region: F32 at offset 64, Q8_0 blocks at offset 64 + 4 * 24
    F = rng.standard_normal((4, 6)).astype(np.float32)
    Wq = (0.05 * rng.standard_normal((3, 32))).astype(np.float32)
    qb = O.q8_0_quantize(Wq)
    region = np.zeros(64 + F.nbytes + qb.nbytes + 16, np.uint8)
    region[64:64 + F.nbytes] = F.view(np.uint8).reshape(-1)
    region[64 + F.nbytes:64 + F.nbytes + qb.nbytes] = qb.reshape(-1)
    assert L.tnn_session_attach_weight_mmap(s, region.ctypes.data, region.nbytes) == 0
    tf = L.tnn_input_2d_persistent_mmap(s, 4, 6, 0, 64)
    tq = L.tnn_input_2d_persistent_mmap(s, 3, 32, 8, 64 + F.nbytes)
    assert tf and tq
    assert not L.tnn_input_1d_persistent_mmap(s, 64, 0, region.nbytes - 8)    # past the region
    assert np.array_equal(g.get(tf), F.astype(np.float64))
    assert np.array_equal(g.get(tq), O.q8_0_dequantize(qb, 32).astype(np.float64))
    # scratch staging: element-wise set, bulk upload, an op, bulk download, statistics
    t = L.tnn_input_2d_f32_persistent(s, 2, 3)
    vals = [1.5, -2.0, 0.25, 4.0, -0.5, 3.0]
    for i, v in enumerate(vals):
        L.tnn_scratch_set(s, i, v)
    assert L.tnn_upload(s, t) == 0
    y = L.tnn_scale(s, t, 2.0)
    L.tnn_set_output(y)
    assert L.tnn_realize(s, y) == 0 and L.tnn_compute(s) == 0
    assert L.tnn_download(s, y) == 0
    assert [L.tnn_scratch_get(s, i) for i in range(6)] == [2 * v for v in vals]
    assert L.tnn_scratch_min_f32(s, 6) == -4.0 and L.tnn_scratch_max_f32(s, 6) == 8.0
    assert L.tnn_scratch_sum_abs_f32(s, 6) == sum(2 * abs(v) for v in vals)
    assert L.tnn_scratch_nan_count_f32(s, 6) == 0
    ti = L.tnn_input_1d_i32_persistent(s, 4)
    for i, v in enumerate([7, -1, 3, 100000]):
        L.tnn_scratch_set_i32(s, i, v)
    assert L.tnn_upload(s, ti) == 0 and L.tnn_download(s, ti) == 0
    assert [L.tnn_scratch_get_i32(s, i) for i in range(4)] == [7, -1, 3, 100000]
    # transposed upload: column j of a row-major (br x bc) matrix -> elements j*br ..
    M = rng.standard_normal((3, 5))
    tt = L.tnn_input_2d_f32_persistent(s, 5, 3)
    assert L.tnn_upload_transposed_f64(s, tt, np.ascontiguousarray(M).ctypes.data_as(C.POINTER(C.c_double)), 3, 5) == 0
    assert rel(g.get(tt), np.float32(M).T) == 0
    assert L.tnn_pin_all_graph_b_nodes(s) == 0
    g.close()


def test_moe_primitives(cuda):
    """tnn_mul_mat_id (f32 and Q8_0 experts, shared and per-slot inputs),
    tnn_add_id, tnn_argsort and tnn_top_k against numpy, ggml semantics
    (tinynn_ggml.h:161-175)."""
    from oracle import oracle as O
    rng = np.random.default_rng(11)
    E, d_in, d_out, nu, T = 4, 64, 48, 2, 5
    W = 0.1 * rng.standard_normal((E, d_out, d_in))
    X = rng.standard_normal((T, 1, d_in))
    Xu = rng.standard_normal((T, nu, d_in))
    ids = rng.integers(0, E, size=(T, nu))
    bias = rng.standard_normal((E, d_out))
    g = Graph()
    L, s = g.L, g.s
    tid = L.tnn_reshape_2d(s, g.i32(ids.reshape(-1)), nu, T)
    wf = g.f32(W)
    y = L.tnn_mul_mat_id(s, wf, g.f32(X), tid)
    yu = L.tnn_mul_mat_id(s, wf, g.f32(Xu), tid)
    # Q8_0 experts: the blocks of every expert row, dequantised for the reference
    blocks = O.q8_0_quantize(W.reshape(E * d_out, d_in).astype(np.float32))
    wq = L.tnn_input_3d_persistent_typed(s, d_in, d_out, E, 8)
    assert wq and L.tnn_upload_q8_0_blocks(s, wq, blocks.ctypes.data, blocks.nbytes) == 0
    Wd = O.q8_0_dequantize(blocks, d_in).reshape(E, d_out, d_in)
    yq = L.tnn_mul_mat_id(s, wq, g.f32(X), tid)
    ya = L.tnn_add_id(s, yu, g.f32(bias), tid)
    v = np.array([[3.0, 1.0, 2.0, 1.0, 5.0, 0.0, 2.0], [1.0, 1.0, 1.0, 0.5, 4.0, 4.0, -1.0]])
    tv = g.f32(v)
    asc, desc, top = L.tnn_argsort(s, tv, 0), L.tnn_argsort(s, tv, 1), L.tnn_top_k(s, tv, 3)
    r_y, r_yu, r_yq, r_ya, r_asc, r_desc, r_top = g.run([y, yu, yq, ya, asc, desc, top])
    ref = np.stack([np.stack([W[ids[t, u]] @ X[t, 0] for u in range(nu)]) for t in range(T)])
    refu = np.stack([np.stack([W[ids[t, u]] @ Xu[t, u] for u in range(nu)]) for t in range(T)])
    refq = np.stack([np.stack([Wd[ids[t, u]] @ X[t, 0] for u in range(nu)]) for t in range(T)])
    assert rel(r_y, ref) < 1e-6 and rel(r_yu, refu) < 1e-6 and rel(r_yq, refq) < 1e-6
    assert rel(r_ya, refu + bias[ids]) < 1e-6
    stable = lambda row, sign: sorted(range(len(row)), key=lambda i: (sign * row[i], i))
    assert np.array_equal(r_asc, [stable(r, 1) for r in v])
    assert np.array_equal(r_desc, [stable(r, -1) for r in v])
    assert np.array_equal(r_top, [stable(r, -1)[:3] for r in v])
    assert L.tnn_mul_mat_id(s, wf, g.f32(rng.standard_normal((T, 3, d_in))), tid) is None   # n_used mismatch
    assert L.tnn_top_k(s, tv, 8) is None
    g.close()


def test_kv_cache_primitives(cuda):
    """tnn_set_rows / tnn_cpy write into their destination's storage, tnn_detach
    is the identity forward, and the causal and cell masks are filled as
    tinynn_ggml.c fills them."""
    rng = np.random.default_rng(12)
    g = Graph()
    L, s = g.L, g.s
    assert L.tnn_null_ptr() is None
    C0 = rng.standard_normal((6, 8))
    R = rng.standard_normal((2, 8))
    Nw = rng.standard_normal((6, 8))
    V = rng.standard_normal((3, 4))
    cache, dst = g.f32(C0), g.f32(np.zeros((6, 8)))
    sr = L.tnn_set_rows(s, cache, g.f32(R), g.i32(np.array([4, 1])))
    cp = L.tnn_cpy(s, g.f32(Nw), dst)
    det = L.tnn_detach(s, g.f32(V))
    r_sr, r_cp, r_det = g.run([sr, cp, det])
    want = C0.copy()
    want[4], want[1] = R[0], R[1]
    assert rel(r_sr, want) < 1e-7 and rel(g.get(cache), want) < 1e-7
    assert rel(r_cp, Nw) < 1e-7 and rel(g.get(dst), Nw) < 1e-7
    assert rel(r_det, V) < 1e-7
    hist, n_tok, pos0 = 7, 3, 4
    m = L.tnn_input_2d_f32_persistent(s, n_tok, hist)
    assert L.tnn_upload_causal_mask(s, m, hist, n_tok, pos0) == 0
    ref = np.array([[0.0 if j <= pos0 + i else -np.inf for j in range(hist)] for i in range(n_tok)])
    assert np.array_equal(g.get(m), ref)
    assert L.tnn_upload_causal_mask(s, m, hist, n_tok, pos0 + 1) == -2
    hi = 5
    cm = L.tnn_input_2d_f32_persistent(s, 2, hi)
    arr = lambda *v: (C.c_long * len(v))(*v)
    owner, cpos = arr(0, 0, -1, 1, -2), arr(0, 3, 1, 0, 0)
    assert L.tnn_upload_cell_mask(s, cm, hi, 2, owner, cpos, arr(0, 1), arr(2, 5), arr(2, 0)) == 0
    vis = [[(o == to and p <= tp) or (o == -1 and p < sh) for o, p in zip([0, 0, -1, 1, -2], [0, 3, 1, 0, 0])]
           for to, tp, sh in ((0, 2, 2), (1, 5, 0))]
    assert np.array_equal(g.get(cm), np.where(vis, 0.0, -np.inf))
    g.close()
