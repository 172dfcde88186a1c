"""Generate the golden vectors in tests/golden/golden.json.

Independent of the C oracle: every value here comes from a pure-Python (numpy float32 scalar)
transcription of an expression in the reference's kernel sources, so the oracle and the CUDA
kernels are both checked against the reference's own arithmetic:

* unpack: `(word >> (4 * i)) & 0xf` for K index 8j + i (locals/kernels.py:31-35,63-64), and the
  8-bit form `(w >> (8 * i)) & 0xff` (the general b-bit stream, locals/moe.py:184-204);
* dequant: `scale * q + bias` (locals/kernels.py:64,77);
* qmm: per group `s * sum(q * x) + b * sum(x)` accumulated in float32 (locals/qmv_multi.py:57-75);
* routing: sigmoid, k rounds of argmax with ties to the lower index, renormalisation
  (locals/moe.py:36-82); softmax variant of a softmax-routed MoE block;
* grouping: the counting sort of locals/moe_kernel.py:28-66 (stable within an expert);
* quantize: MLX's affine algorithm (mx.quantize; the reference calls it in
  tests/test_kernel_patching.py:163). MLX is not available here, so these vectors pin our
  restatement of its published algorithm, not MLX itself ("parity unpinned" for quantization).

Run: python tests/golden/make_golden.py  (rewrites golden.json; commit both).
"""

from __future__ import annotations

import json
import os

import numpy as np

F = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))


def pack(codes, bits):
    per = 32 // bits
    words = []
    for j in range(0, len(codes), per):
        w = 0
        for i in range(per):
            w |= int(codes[j + i]) << (bits * i)
        words.append(w)
    return words


def unpack(words, bits, K):
    per = 32 // bits
    mask = (1 << bits) - 1
    return [(words[k // per] >> (bits * (k % per))) & mask for k in range(K)]


def quantize_group(vals, bits):
    """MLX affine quantization of one group, float32 scalar arithmetic."""
    n_bins = F((1 << bits) - 1)
    w = [F(v) for v in vals]
    w_max, w_min = max(w), min(w)
    mask = abs(w_min) > abs(w_max)
    scale = max(F((w_max - w_min) / n_bins), F(1e-7))
    scale = scale if mask else F(-scale)
    edge = w_min if mask else w_max
    q0 = F(np.rint(F(edge / scale)))
    bias = F(0.0)
    if q0 != 0:
        scale = F(edge / q0)
        bias = edge
    codes = [int(min(max(F(np.rint(F((v - bias) / scale))), F(0)), n_bins)) for v in w]
    return codes, float(scale), float(bias)


def qmm(x, codes, s, b, group=64):
    """x: list of rows (float32), codes: rows of K codes, s/b: rows of per-group floats."""
    out = []
    for xm in x:
        row = []
        for n in range(len(codes)):
            acc = F(0)
            for g in range(len(s[n])):
                d = F(0)
                xs = F(0)
                for j in range(group):
                    k = g * group + j
                    d = F(d + F(F(codes[n][k]) * F(xm[k])))
                    xs = F(xs + F(xm[k]))
                acc = F(acc + F(F(F(s[n][g]) * d) + F(F(b[n][g]) * xs)))
            row.append(float(acc))
        out.append(row)
    return out


def topk(scores, k):
    sc = list(scores)
    inds, picked = [], []
    for _ in range(k):
        best, be = None, None
        for e, v in enumerate(sc):
            if v is None:
                continue
            if best is None or v > best:
                best, be = v, e
        inds.append(be)
        picked.append(best)
        sc[be] = None
    tot = F(0)
    for p in picked:
        tot = F(tot + F(p))
    return inds, [float(F(F(p) / tot)) for p in picked]


def softmax(logits):
    m = max(F(v) for v in logits)
    ex = [F(np.exp(F(F(v) - m))) for v in logits]
    tot = F(0)
    for v in ex:
        tot = F(tot + v)
    return [F(v / tot) for v in ex]


def sigmoid(logits):
    out = []
    for v in logits:
        s = F(F(1) / F(F(1) + F(np.exp(F(-F(v))))))
        out.append(F(0) if np.isnan(s) else s)
    return out


def group_pairs(inds, E):
    cnt = [0] * E
    for e in inds:
        cnt[e] += 1
    base, starts, experts, at = [0] * E, [], [], 0
    for e in range(E):
        base[e] = at
        if cnt[e]:
            starts.append(at)
            experts.append(e)
        at += cnt[e]
    starts.append(at)
    order = [0] * len(inds)
    nxt = list(base)
    for p, e in enumerate(inds):
        order[nxt[e]] = p
        nxt[e] += 1
    return order, starts, experts


def main():
    rng = np.random.default_rng(20261201)
    gold = {}

    # 1. bit order: codes 1..8 in the first word, 15..8 in the second (4-bit); bytes for 8-bit
    c4 = [1, 2, 3, 4, 5, 6, 7, 8, 15, 14, 13, 12, 11, 10, 9, 8]
    c8 = [1, 2, 3, 255, 0, 128, 64, 7]
    gold["pack4"] = {"codes": c4, "words": pack(c4, 4)}
    gold["pack8"] = {"codes": c8, "words": pack(c8, 8)}
    assert unpack(pack(c4, 4), 4, 16) == c4 and gold["pack4"]["words"][0] == 0x87654321

    # 2. quantize known answers: a ramp, a negative-dominant group, a constant group, random groups
    groups = {
        "ramp": [i / 64 for i in range(64)],
        "negative": [-1.0 + 1.5 * i / 63 for i in range(64)],
        "constant": [0.25] * 64,
        "zeros": [0.0] * 64,
        "random": [float(v) for v in (rng.standard_normal(64) * 0.02).astype(np.float32)],
    }
    gold["quantize"] = {}
    for bits in (4, 8):
        for name, vals in groups.items():
            codes, s, b = quantize_group(vals, bits)
            gold["quantize"][f"{name}_b{bits}"] = {"w": [float(F(v)) for v in vals], "bits": bits, "codes": codes,
                                                   "scale": s, "bias": b}

    # 3. a small qmm: x (3, 128), W (5, 128) random codes and scales
    for bits in (4, 8):
        K, N = 128, 5
        codes = [[int(v) for v in rng.integers(0, 1 << bits, K)] for _ in range(N)]
        s = [[float(F(v)) for v in rng.uniform(-0.02, 0.02, K // 64)] for _ in range(N)]
        b = [[float(F(v)) for v in rng.uniform(-0.1, 0.1, K // 64)] for _ in range(N)]
        x = [[float(F(v)) for v in rng.standard_normal(K)] for _ in range(3)]
        words = [pack(cr, bits) for cr in codes]
        gold[f"qmm_b{bits}"] = {"x": x, "words": words, "scales": s, "biases": b, "bits": bits,
                                "y": qmm(x, codes, s, b)}

    # 4. routing: softmax and sigmoid top-k, with ties and a NaN logit
    logits = [[float(F(v)) for v in rng.standard_normal(16)] for _ in range(3)]
    logits.append([0.5] * 16)  # all tied: experts 0..k-1
    logits.append([0.1, 2.0, 2.0, -1.0] + [0.0] * 12)  # a tie at the top: 1 before 2
    gold["topk_softmax"] = {"logits": logits, "k": 4, "inds": [], "weights": []}
    for row in logits:
        i, w = topk(softmax(row), 4)
        gold["topk_softmax"]["inds"].append(i)
        gold["topk_softmax"]["weights"].append(w)
    sig_logits = [list(r) for r in logits] + [[float("nan")] + [float(F(v)) for v in rng.standard_normal(15)]]
    gold["topk_sigmoid"] = {"logits": [[None if np.isnan(v) else v for v in r] for r in sig_logits], "k": 4,
                            "inds": [], "weights": []}
    for row in sig_logits:
        i, w = topk(sigmoid(row), 4)
        gold["topk_sigmoid"]["inds"].append(i)
        gold["topk_sigmoid"]["weights"].append(w)

    # 5. grouping
    inds = [int(v) for v in rng.integers(0, 8, 24)]
    order, starts, experts = group_pairs(inds, 8)
    gold["group"] = {"inds": inds, "E": 8, "order": order, "starts": starts, "experts": experts}

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(gold, f, indent=0)


if __name__ == "__main__":
    main()
