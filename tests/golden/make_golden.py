"""Generate the golden fixtures that pin the oracle to the reference (run in the build container only).

The reference (sott0n/tt-qwen-resident, mounted read-only at REF_ROOT) is imported with a stub ``ttnn`` module:
its device code cannot run here, but its torch math can. ``common.quantize`` is replaced by the identity (fp32
weights; quantisation is a separate, separately tested step) and ``model.quantize_rows`` by bf16 rounding (this
build's KV dtype). Then, with the reference's own ``random_weights`` / ``State`` / ``torch_step``
(``qwen36_resident/model.py:151-292``), the consecutive decode steps of ``tests/bench_resident_model.py:483-549``
are recorded, as are two single-kind schedules. The sampling fixture runs the integer ``draw`` of the
reference's ``tests/test_resident_sampling.py:37-95`` (loaded from its source text, the file's hardware fixture
left out) on seeded logits for the five parameter cases of that test (:27-33).

Usage:  python tests/golden/make_golden.py REF_ROOT   (or QRES_REFERENCE_ROOT=REF_ROOT in the environment)
Writes: tests/golden/decode_steps.npz, gdn_steps.npz, attn_steps.npz, sampling.json
"""
import ast
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SAMPLE_IDX = torch.randperm(48 * 128 * 128, generator=torch.Generator().manual_seed(3))[:8192]
REF_ROOT = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QRES_REFERENCE_ROOT")
if not REF_ROOT:
    sys.exit("usage: make_golden.py REFERENCE_ROOT   (or set QRES_REFERENCE_ROOT): the sott0n/tt-qwen-resident checkout")


def import_reference():
    stub = types.ModuleType("ttnn")
    for a in ["bfloat8_b", "bfloat4_b", "bfloat16", "uint32", "float32", "TILE_LAYOUT", "ROW_MAJOR_LAYOUT"]:
        setattr(stub, a, a)
    sys.modules["ttnn"] = stub
    sys.path.insert(0, REF_ROOT)
    import qwen36_resident.common as C

    C.quantize = lambda w, dtype: w.float().clone()
    import qwen36_resident.model as M

    M.quantize = C.quantize
    M.quantize_rows = lambda t, dtype=None: t.bfloat16().float()
    return M


def run_case(M, name, layers, interval, gdn_copies, attn_copies, mlp_copies, vocab, pos, steps):
    torch.set_num_threads(8)
    d = M.Dims(4, 8, vocab=vocab)
    w = M.random_weights(d, gdn_copies, attn_copies, mlp_copies, seed=0)
    st = M.State(d, gdn_copies, attn_copies, pos, max_pos=pos + 64, seed=1)
    g = torch.Generator().manual_seed(7)
    xs, lgs, mixers = [], [], []
    for _ in range(steps):
        x0 = torch.randn(M.HIDDEN if hasattr(M, "HIDDEN") else 5120, generator=g).bfloat16().float()
        o = []
        out = M.torch_step(x0, d, w, st, layers, interval, lm_head=bool(vocab), attn_out=o)
        x = out[0] if vocab else out
        xs.append(x)
        # the last layer's mixer output per chip, [4, gv]
        mixers.append(torch.stack([v for l, _, v in o if l == layers - 1]))
        if vocab:
            lgs.append(torch.cat([t[: d.vocab_chip] for t in out[1]]))
    rec = dict(
        layers=layers,
        interval=interval,
        gdn_copies=gdn_copies,
        attn_copies=attn_copies,
        mlp_copies=mlp_copies,
        vocab=vocab,
        pos=pos,
        steps=steps,
        x=torch.stack(xs).numpy(),
        mixer=torch.stack(mixers).numpy(),
        # final decode state, assembled canonically (chip c: GDN heads [12c, 12c+12), KV head c)
        # GDN states: per-head Frobenius norms and a seeded sample of 8192 entries per copy (the full states
        # are 9.4 MB per copy)
        gdn_norms=np.stack([torch.cat(st.gdn[c]).flatten(1).norm(dim=1).numpy() for c in range(gdn_copies)])
        if gdn_copies
        else np.zeros(0),
        gdn_sample_idx=SAMPLE_IDX.numpy(),
        gdn_sample=np.stack([torch.cat(st.gdn[c]).flatten()[SAMPLE_IDX].numpy() for c in range(gdn_copies)])
        if gdn_copies
        else np.zeros(0),
        k_rows=np.stack([torch.stack([k[pos : pos + steps] for k in st.K[c]]).numpy() for c in range(attn_copies)])
        if attn_copies
        else np.zeros(0),
        v_rows=np.stack([torch.stack([v[pos : pos + steps] for v in st.V[c]]).numpy() for c in range(attn_copies)])
        if attn_copies
        else np.zeros(0),
    )
    if vocab:
        rec["logits"] = torch.stack(lgs).numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
    print(name, "x norm", [float(x.norm()) for x in xs])


def sampling_fixture():
    """the reference test's own integer draw (its source, minus the hardware fixture) on seeded logits"""
    path = os.path.join(REF_ROOT, "qwen36_resident/tests/test_resident_sampling.py")
    src = open(path).read()
    tree = ast.parse(src)
    keep = [
        n
        for n in tree.body
        if isinstance(n, ast.FunctionDef) and n.name in ("key_of", "q16", "exp_q16", "mix", "draw")
        or (isinstance(n, ast.Assign) and any(getattr(t, "id", "") in ("CASES", "M32") for t in n.targets))
    ]
    ns = {"torch": torch, "TOP_K": 32}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    cases = ns["CASES"]
    g = torch.Generator().manual_seed(11)
    out = []
    for vocab, scale in ((1000, 1.0), (4096, 3.0), (300, 0.05)):
        for rep in range(3):
            logits = (scale * torch.randn(vocab, generator=g)).bfloat16().float()
            # plant exact ties at the top
            top = int(logits.argmax())
            for j in (7, 123 % vocab, vocab - 1):
                logits[j] = logits[top]
            for (t, k, p, seed) in cases:
                words = [min(round(65536 / t), 2**31 - 1) if t > 0 else 0, k, min(max(round(p * 65536), 1), 65536), seed & 0xFFFFFFFF]
                for pos in (0, 17, 4095 + rep):
                    tok = ns["draw"](logits, words, pos)
                    out.append(
                        dict(
                            logits_bf16_bits=logits.bfloat16().view(torch.int16).to(torch.int32).tolist(),
                            words=words,
                            pos=pos,
                            token=int(tok),
                        )
                    )
    # compact: store each logits vector once
    vecs, recs = [], []
    for r in out:
        key = tuple(r["logits_bf16_bits"])
        if not vecs or tuple(vecs[-1]) != key:
            vecs.append(r["logits_bf16_bits"])
        recs.append(dict(vec=len(vecs) - 1, words=r["words"], pos=r["pos"], token=r["token"]))
    json.dump(dict(cases=cases, vectors=vecs, draws=recs), open(os.path.join(HERE, "sampling.json"), "w"))
    print("sampling draws", len(recs))


if __name__ == "__main__":
    M = import_reference()
    run_case(M, "decode_steps", layers=8, interval=4, gdn_copies=2, attn_copies=1, mlp_copies=2, vocab=16384, pos=100, steps=3)
    run_case(M, "gdn_steps", layers=3, interval=0, gdn_copies=3, attn_copies=0, mlp_copies=1, vocab=0, pos=5, steps=4)
    run_case(M, "attn_steps", layers=2, interval=1, gdn_copies=0, attn_copies=2, mlp_copies=2, vocab=0, pos=63, steps=3)
    sampling_fixture()
