"""Generate the committed golden fixtures in this folder.

Run in a container that has the reference tree and gguf-py:
    python tests/golden/make_golden.py

Sources (all paths inside the reference project):
  * op_smokes.json — the inputs of the reference's op-level A/B smokes and the
    values their own pure-Ruby reference functions compute on those inputs,
    restated line by line in Python below:
      tinynn/ab_smoke_adamw_op.rb:11-31,37-56   (adam_native)
      tinynn/ab_smoke_cegrad.rb:9-66            (cross_entropy_grad_native)
      tinynn/ab_smoke_silu_back.rb:12-46        (silu_back_native)
      tinynn/ab_smoke_rms_norm.rb:9-41          (rms_norm_native)
      tinynn/ab_smoke_softmax.rb                (softmax_native)
      tinynn/ab_smoke_back.rb                   (softmax_back_native)
    plus the recorded known answer of tinynn/rms_norm_back_probe.c:11-18
    (x = dz = [1,0,0,0], eps = 1e-4 -> [0.0008, 0, 0, 0]).
  * q8_0.npz — Q8_0 blocks produced by gguf-py's quantizer (gguf/quants.py
    class Q8_0), the quantizer prep/convert_smollm2_to_gguf.py uses, on seeded
    inputs including zero blocks and half-way ties.
  * lcg.json — the init streams of lib/toy/llm/engine/llama_seq_engine.rb
    (lcg_seed_state :1416-1428, lcg_uniform! :1409-1414, upload_gaussian
    :1383-1407, upload_lora_q_init! :2545-2575) restated with Python's exact
    big integers and libm, independently of the C oracle.
"""
import json
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def adam_native(param, grad, m, v, lr, b1, b2, eps, omc1, omc2):
    np_, nm, nv = [], [], []
    for i in range(len(param)):
        gi = grad[i]
        new_m = b1 * m[i] + (1.0 - b1) * gi
        new_v = b2 * v[i] + (1.0 - b2) * gi * gi
        nm.append(new_m)
        nv.append(new_v)
        m_hat = new_m / omc1
        v_hat = new_v / omc2
        np_.append(param[i] - lr * m_hat / (math.sqrt(v_hat) + eps))
    return np_, nm, nv


def softmax_native(rows):
    out = []
    for r in rows:
        m = r[0]
        for v in r[1:]:
            if v > m:
                m = v
        e = [math.exp(v - m) for v in r]
        s = 0.0
        for x in e:
            s = s + x
        out.append([x / s for x in e])
    return out


def op_smokes():
    g = {}
    n = 12
    param = [i * 0.1 - 0.5 for i in range(n)]
    grad = [(i - 6.0) * 0.05 for i in range(n)]
    mst = [i * 0.02 for i in range(n)]
    vst = [i * 0.01 for i in range(n)]
    lr, b1, b2, eps = 0.001, 0.9, 0.999, 1.0e-8
    omc1, omc2 = 1.0 - 0.9, 1.0 - 0.999
    p2, m2, v2 = adam_native(param, grad, mst, vst, lr, b1, b2, eps, omc1, omc2)
    g["adamw"] = dict(shape=[3, 4], param=param, grad=grad, m=mst, v=vst,
                      hp=[lr, b1, b2, eps, 0.0, 1.0 / omc1, 1.0 / omc2],
                      want_param=p2, want_m=m2, want_v=v2, tol_param=1.0e-4, tol_mv=1.0e-5,
                      source="tinynn/ab_smoke_adamw_op.rb")
    logits = [[(r * 5 + c) * 0.3 - 2.0 for c in range(5)] for r in range(3)]
    targets = [4, 0, 2]
    sm = softmax_native(logits)
    want = [[(sm[i][v] - (1.0 if v == targets[i] else 0.0)) * (1.0 / 3) for v in range(5)] for i in range(3)]
    g["ce_grad"] = dict(logits=logits, targets=targets, want=want, tol=1.0e-4, source="tinynn/ab_smoke_cegrad.rb")
    xs = [0.0, 0.5, 2.5, -0.3, -1.2, 4.0, 0.01, -3.5]
    dys = [1.0, -0.5, 2.0, -1.0, 0.3, 0.7, -2.0, 0.5]
    want = []
    for x, dy in zip(xs, dys):
        s = 1.0 / (1.0 + math.exp(-x))
        want.append(dy * (s * (1.0 + x * (1.0 - s))))
    g["silu_back"] = dict(x=xs, dy=dys, want=want, tol=1.0e-3, source="tinynn/ab_smoke_silu_back.rb")
    x = [[1.0, 2.0, -1.0, 0.5], [-0.5, 3.0, 0.0, 1.5]]
    gamma = [1.0, 0.5, 2.0, 1.5]
    eps = 0.00001
    want = []
    for r in x:
        ss = 0.0
        for v in r:
            ss = ss + v * v
        rms = math.sqrt(ss / 4.0 + eps)
        want.append([r[c] / rms * gamma[c] for c in range(4)])
    g["rms_norm"] = dict(x=x, gamma=gamma, eps=eps, want=want, tol=1.0e-3, source="tinynn/ab_smoke_rms_norm.rb")
    x = [[1.0, 2.0, 3.0, 4.0], [0.5, 0.5, 0.5, 0.5]]
    g["softmax"] = dict(x=x, want=softmax_native(x), tol=1.0e-5, source="tinynn/ab_smoke_softmax.rb")
    xsm = [[(r * 4 + c) * 0.4 - 2.0 for c in range(4)] for r in range(3)]
    dysm = [[(r * 4 + c) * 0.2 - 1.0 for c in range(4)] for r in range(3)]
    a = softmax_native(xsm)
    want = []
    for r in range(3):
        dot = 0.0
        for c in range(4):
            dot = dot + a[r][c] * dysm[r][c]
        want.append([a[r][c] * (dysm[r][c] - dot) for c in range(4)])
    g["softmax_back"] = dict(x=xsm, dy=dysm, want=want, tol=1.0e-3, source="tinynn/ab_smoke_back.rb")
    g["rms_norm_back_known"] = dict(x=[1.0, 0.0, 0.0, 0.0], dz=[1.0, 0.0, 0.0, 0.0], eps=1.0e-4,
                                    want=[0.0008, 0.0, 0.0, 0.0], tol=1.0e-6,
                                    source="tinynn/rms_norm_back_probe.c:11-18")
    return g


def q8_fixture():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as QT
    rng = np.random.default_rng(1234)
    a = (rng.standard_normal((16, 64)) * 0.02).astype(np.float32)      # weight-like
    b = rng.standard_normal((8, 96)).astype(np.float32)                 # unit gaussian
    c = np.zeros((2, 32), np.float32)                                   # all-zero blocks
    c[1, :] = 0.0
    c[1, 3] = 1e-30                                                     # tiny amax -> fp16 subnormal/zero d
    d = np.zeros((1, 32), np.float32)                                   # exact half-way ties: x*id = k + 0.5
    d[0, 0] = 127.0
    d[0, 1:] = np.arange(31, dtype=np.float32) + np.float32(0.5)
    e = (rng.standard_normal((4, 576)) * 3.0).astype(np.float32)        # SmolLM2 row width
    out = {}
    for name, x in (("a", a), ("b", b), ("c", c), ("d", d), ("e", e)):
        out[name + "_x"] = x
        out[name + "_q"] = quants.quantize(x, QT.Q8_0)
        out[name + "_dq"] = quants.dequantize(out[name + "_q"], QT.Q8_0).astype(np.float32)
    return out


def lcg_fixture():
    def seed_state(seed):
        s = ((seed + 104729) * 2654435761) % 2147483647
        if s <= 0:
            s = seed + 104729
        for _ in range(8):
            s = (s * 1103515245 + 12345) & 0x7FFFFFFF
        return s

    def gaussian(state, n, std):
        out, pair, saved = [], 0, 0.0
        s = state
        for _ in range(n):
            if pair == 0:
                s = (s * 1103515245 + 12345) & 0x7FFFFFFF
                u1 = (s + 1.0) / 2147483648.0
                s = (s * 1103515245 + 12345) & 0x7FFFFFFF
                u2 = (s + 1.0) / 2147483648.0
                if u1 < 1.0e-300:
                    u1 = 1.0e-300
                r = math.sqrt(-2.0 * math.log(u1))
                th = 2.0 * math.pi * u2
                out.append(r * math.cos(th) * std)
                saved = r * math.sin(th) * std
                pair = 1
            else:
                out.append(saved)
                pair = 0
        return out, s

    def lora_a(s, n, init_scale):
        out = []
        for _ in range(n):
            s = (s * 1103515245 + 12345) & 0x7FFFFFFF
            u1 = (s + 1.0) / 2147483648.0
            s = (s * 1103515245 + 12345) & 0x7FFFFFFF
            u2 = (s + 1.0) / 2147483648.0
            out.append(init_scale * math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * u2))
        return out, s

    res = {"seed_state": {str(sd): seed_state(sd) for sd in (0, 1, 42, 12345, 2147483646)}}
    st = seed_state(42)
    g1, st1 = gaussian(st, 33, 0.02)
    g2, st2 = gaussian(st1, 16, 1.0)
    res["gaussian_seed42"] = dict(n1=33, std1=0.02, n2=16, std2=1.0, values1=[float(np.float32(v)) for v in g1],
                                  values2=[float(np.float32(v)) for v in g2], state_after=st2)
    la, sla = lora_a(42, 24, 0.01)
    res["lora_a_seed42"] = dict(n=24, init_scale=0.01, values=[float(np.float32(v)) for v in la], state_after=sla)
    return res


if __name__ == "__main__":
    with open(os.path.join(HERE, "op_smokes.json"), "w") as f:
        json.dump(op_smokes(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "q8_0.npz"), **q8_fixture())
    with open(os.path.join(HERE, "lcg.json"), "w") as f:
        json.dump(lcg_fixture(), f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))
