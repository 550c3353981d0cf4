"""Order keys, argmax / top-k rules and the integer sampling draw (TEST INFRASTRUCTURE ONLY).

Restates ``qwen36_resident/kernels/sampling.hpp`` (key_of / bf16_of :24-25, the tie rule ``better`` :27,
``merge`` :53-74, ``q16`` :77-86, ``exp_q16`` :89-101, ``mix`` :103-110, ``draw`` :113-143) and the host
argmax rule of ``model.py:1558-1573`` (largest logit, the smallest vocab index on ties), in Python integers.
These are bit-exact contracts: the GPU's candidates, lists and draws must equal them exactly.
"""
import torch

TOP_K = 32
M32 = 0xFFFFFFFF


def key_of(b):
    """bf16 bits -> unsigned key ordered like the values"""
    return (~b & 0xFFFF) if b & 0x8000 else (b | 0x8000)


def bf16_of(key):
    return (key & 0x7FFF) if key & 0x8000 else (~key & 0xFFFF)


def keys_of(logits):
    """tensor of logits (any float) -> int64 keys of their bf16 values"""
    bits = logits.to(torch.bfloat16).view(torch.int16).to(torch.int64) & 0xFFFF
    return torch.where(bits & 0x8000 != 0, ~bits & 0xFFFF, bits | 0x8000)


def better(k, i, bk, bi):
    return k > bk or (k == bk and i < bi)


def argmax_rule(logits):
    """vocab index of the largest bf16 logit, the smallest index on ties"""
    keys = keys_of(logits.flatten())
    best = int(keys.max())
    return int(torch.nonzero(keys == best)[0, 0])


def topk_list(logits, k=TOP_K, base=0):
    """the top-k (key, index) list of a logits vector: keys descending, the smaller index first on equal keys;
    unused entries key 0, index 0xffffffff (sampling.hpp clear)"""
    keys = keys_of(logits.flatten())
    n = keys.numel()
    order = sorted(range(n), key=lambda i: (-int(keys[i]), i))[:k]
    ks = [int(keys[i]) for i in order] + [0] * (k - len(order))
    ix = [base + i for i in order] + [M32] * (k - len(order))
    return ks, ix


def merge(lists, k=TOP_K):
    """sampling.hpp merge: the top k of several (keys, indices) lists"""
    heads = [0] * len(lists)
    out_k, out_i = [], []
    for _ in range(k):
        best, bk, bi = None, 0, 0
        for s, (ks, ix) in enumerate(lists):
            if heads[s] == k:
                continue
            kk, ii = ks[heads[s]], ix[heads[s]]
            if best is None or better(kk, ii, bk, bi):
                best, bk, bi = s, kk, ii
        out_k.append(bk)
        out_i.append(bi)
        heads[best] += 1
    return out_k, out_i


def q16(b):
    e = (b >> 7) & 0xFF
    if e == 0:
        return 0
    m = (b & 0x7F) | 0x80
    shift = e - 118
    v = (m << 22 if shift > 22 else m << shift) if shift >= 0 else (0 if shift < -31 else m >> -shift)
    return -v if b & 0x8000 else v


def exp_q16(d):
    t = (d * 94548) >> 16
    n, f = t >> 16, t & 0xFFFF
    p = 87
    for c in (630, 3638, 15743, 45426, 65536):
        p = c + (((p * f) & M32) >> 16)
    return 0 if n <= -31 else p >> -n


def mix(x):
    x &= M32
    x ^= x >> 16
    x = (x * 0x7FEB352D) & M32
    x ^= x >> 15
    x = (x * 0x846CA68B) & M32
    return x ^ (x >> 16)


def sampling_words(temperature=0.0, top_k=1, top_p=1.0, seed=0):
    """model.py:1528-1536: [1/T in Q16 (0 = greedy), top_k (<1: TOP_K), top_p in Q16, seed]"""
    top_k = TOP_K if top_k < 1 else min(int(top_k), TOP_K)
    inv = min(round(65536 / temperature), 2**31 - 1) if temperature > 0 else 0
    return [inv, top_k, min(max(round(top_p * 65536), 1), 65536), int(seed) & M32]


def draw(list_keys, list_idx, words, pos):
    """sampling::draw over a global top-k list"""
    inv_temp, top_k, top_p, seed = (int(v) for v in words[:4])
    k = min(top_k, TOP_K)
    if inv_temp == 0 or k <= 1:
        return list_idx[0]
    l0 = q16(bf16_of(list_keys[0]))
    w = []
    for i in range(k):
        d = max(((q16(bf16_of(list_keys[i])) - l0) * inv_temp) >> 16, -(64 << 16))
        w.append(exp_q16(d) if list_keys[i] else 0)
    total = sum(w) & M32
    limit = (total * top_p) >> 16
    kept, mass = 0, 0
    while kept < k and (kept == 0 or mass < limit):
        mass += w[kept]
        kept += 1
    target = (mix(seed ^ mix((pos + 0x9E3779B9) & M32)) * mass) >> 32
    for i in range(kept):
        if target < w[i]:
            return list_idx[i]
        target -= w[i]
    return list_idx[kept - 1]
