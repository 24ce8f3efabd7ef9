"""Independent numpy restatements used to check the C oracle on CPU.

These are written from the reference's formulas (kernels/*.cuh and
kernels/unit_tests/run_tests.cu) in float64 with fp16 rounding at the same
store points; the C oracle must agree with them within the stated bounds.
"""
import numpy as np


def h(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16)


def rmsnorm(x, w, eps=1e-6):
    xf = x.astype(np.float64)
    r = 1.0 / np.sqrt(np.mean(xf * xf) + eps)
    return h((x.astype(np.float32) * np.float32(r)) * w.astype(np.float32))


def rope_cache(qkv, kc, vc, pos, nh=16, hd=128):
    qkv, kc, vc = qkv.copy(), kc.copy(), vc.copy()
    H = nh * hd
    t = np.arange(hd // 2)
    theta = pos * np.power(10000.0, -2.0 * t / hd)
    c, s = np.cos(theta), np.sin(theta)
    for hh in range(nh):
        i1 = hh * hd + t
        i2 = i1 + hd // 2
        q1, q2 = qkv[i1].astype(np.float64), qkv[i2].astype(np.float64)
        k1, k2 = qkv[H + i1].astype(np.float64), qkv[H + i2].astype(np.float64)
        qkv[i1], qkv[i2] = h(q1 * c - q2 * s), h(q2 * c + q1 * s)
        kc[pos * H + i1], kc[pos * H + i2] = h(k1 * c - k2 * s), h(k2 * c + k1 * s)
        vc[pos * H + i1], vc[pos * H + i2] = qkv[2 * H + i1], qkv[2 * H + i2]
    return qkv, kc, vc


def attention(q, K, V, L, stride, hd=128):
    """softmax(q K^T / sqrt(hd)) V over rows [0, L) (float64)."""
    Kr = np.stack([K[i * stride: i * stride + hd] for i in range(L)]).astype(np.float64)
    Vr = np.stack([V[i * stride: i * stride + hd] for i in range(L)]).astype(np.float64)
    s = Kr @ q[:hd].astype(np.float64) / np.sqrt(hd)
    p = np.exp(s - s.max())
    p /= p.sum()
    return p @ Vr


def argmax_reference(logits):
    """Step-by-step simulation of kernels/argmax.cuh:7-72 with blockDim 512."""
    V = logits.size
    T = 512
    ipt = (V + T - 1) // T
    vals = logits.astype(np.float32)
    lv = np.full(T, -np.inf, np.float32)
    li = np.full(T, -1, np.int64)
    for t in range(T):
        for i in range(ipt):
            idx = t * ipt + i
            if idx < V and vals[idx] > lv[t]:
                lv[t], li[t] = vals[idx], idx

    def butterfly(v, ix):
        v, ix = v.copy(), ix.copy()
        for mask in (16, 8, 4, 2, 1):
            nv, ni = v.copy(), ix.copy()
            for lane in range(32):
                p = lane ^ mask
                if v[p] > v[lane]:
                    nv[lane], ni[lane] = v[p], ix[p]
            v, ix = nv, ni
        return v[0], ix[0]

    wv = np.full(32, -np.inf, np.float32)
    wi = np.full(32, -1, np.int64)
    for w in range(T // 32):
        wv[w], wi[w] = butterfly(lv[w * 32:(w + 1) * 32], li[w * 32:(w + 1) * 32])
    return int(butterfly(wv, wi)[1])


def model_step(W, kc, vc, token, pos, cfg, eps=1e-6):
    """float64 forward of one decode step with fp16 stores (qwen_infer.cu:614-737).
    W: dict of [N,K] fp16 matrices as in the .bin; kc/vc [layers, S, H] fp16 (mutated)."""
    H, NH, IM = cfg["hidden_size"], cfg["num_heads"], cfg["intermediate_size"]
    x = W["wte"][token].copy()
    for l in range(cfg["num_layers"]):
        L = W["layers"][l]
        xn = rmsnorm(x, L["ln1"], eps)
        qkv = h(L["qkv_w"].astype(np.float64) @ xn.astype(np.float64))
        qkv = h(qkv.astype(np.float32) + L["qkv_b"].astype(np.float32))
        kcl, vcl = kc[l].reshape(-1), vc[l].reshape(-1)
        qkv, kcl2, vcl2 = rope_cache(qkv, kcl, vcl, pos, NH, 128)
        kc[l] = kcl2.reshape(kc[l].shape)
        vc[l] = vcl2.reshape(vc[l].shape)
        att = np.zeros(H, np.float16)
        for hh in range(NH):
            att[hh * 128:(hh + 1) * 128] = h(attention(qkv[hh * 128:], kc[l].reshape(-1)[hh * 128:],
                                                       vc[l].reshape(-1)[hh * 128:], pos + 1, H))
        o = h(L["proj_w"].astype(np.float64) @ att.astype(np.float64))
        x = h(x.astype(np.float32) + o.astype(np.float32))
        xn = rmsnorm(x, L["ln2"], eps)
        a = h(L["w1"].astype(np.float64) @ xn.astype(np.float64)).astype(np.float32)
        b = h(L["w2"].astype(np.float64) @ xn.astype(np.float64)).astype(np.float32)
        act = h(a * (b / (1.0 + np.exp(-b))))
        c = h(L["cproj"].astype(np.float64) @ act.astype(np.float64))
        x = h(x.astype(np.float32) + c.astype(np.float32))
    xn = rmsnorm(x, W["ln_f"], eps)
    logits = h(W["lm_head"].astype(np.float64) @ xn.astype(np.float64))
    return logits, x


def read_bin(path):
    """Parse a QWDF .bin (model_weights/convert_weights.py:107-185) into numpy arrays."""
    with open(path, "rb") as f:
        hdr = np.frombuffer(f.read(28), dtype="<u4")
        magic, V, H, NL, NH, IM, S = (int(v) for v in hdr)
        assert magic == 0x46445751

        def rd(*shape):
            n = int(np.prod(shape))
            return np.frombuffer(f.read(2 * n), dtype=np.float16).reshape(shape)
        W = {"wte": rd(V, H), "layers": []}
        for _ in range(NL):
            W["layers"].append(dict(ln1=rd(H), qkv_w=rd(3 * H, H), qkv_b=rd(3 * H), proj_w=rd(H, H), ln2=rd(H),
                                    w1=rd(IM, H), w2=rd(IM, H), cproj=rd(H, IM)))
        W["ln_f"] = rd(H)
        W["lm_head"] = rd(V, H)
    cfg = dict(vocab_size=V, hidden_size=H, num_layers=NL, num_heads=NH, intermediate_size=IM, max_seqlen=S)
    return W, cfg
