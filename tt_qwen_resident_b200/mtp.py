"""Greedy speculative decode with the MTP draft layer on B200: sott0n/tt-qwen-resident's ``SpecDecoder``
(qwen36_resident/mtp.py:292-591) over two ``ResidentModel`` contexts, generalised from one draft per step to K
(BASELINE: 3 drafts, a 4-row verify step).

The main model runs the verify step (ResidentModel(verify=True), rows = K + 1 consecutive positions of one user,
row r sees rows < r): row 0 holds the last committed token t at position p, rows 1..K the drafts d_1..d_K. Its
greedy picks a_0..a_K accept the drafts up to the first mismatch: with k = the number of leading r with
a_r == d_(r+1), the step commits a_0..a_k (k accepted drafts and one more token) and the next step continues from
row k (position p + k + 1, state slot (slot + k) % R; nothing is rolled back: the conv history and the KV cache
are position-keyed and each row left its GDN state in its own slot). Every committed token is the main model's
greedy pick at its position, so the output equals plain greedy decode token for token (``greedy``).

The draft model is one attention decoder layer with its own KV cache and the main model's lm_head; its entry at
position q takes x0 = fc([rmsnorm(embed(tok[q + 1])) | rmsnorm(h_q)]) for the main model's last x h_q at q and
predicts tok[q + 2] (mtp.py:1-14). After a main step at p it adds the entries q = p .. p + k of the committed path
(the main model's rows as h, the committed tokens), which keeps its KV cache that of the committed sequence; the
last of them drafts d'_1, and K - 1 chained entries (each on the previous draft's token and last x) draft the rest.
Host driven, as the reference's ``generate``: each step's picks are read back before the next step is written.
"""
import time

import torch

from .model import ResidentModel


class SpecDecoder:
    def __init__(self, main, draft, drafts=3):
        """main: ResidentModel(verify=True, batch=drafts + 1, lm_head, embed); draft: ResidentModel with the fc
        (fc=...), one attention layer, batch 1, the same lm_head and embedding"""
        assert main.verify and main.batch == drafts + 1 and main.lm_head and main.embed is not None
        assert draft.w_fc is not None and draft.batch == 1 and draft.lm_head and draft.embed is not None
        self.main, self.draft, self.K = main, draft, drafts
        self.R = drafts + 1
        self.draft_fn = None  # tests: replace the draft model by a function (seq, p, K) -> K drafts

    # ------------------------------------------------------------------------------------------ device steps
    def _main(self, toks, p, slot):
        m = self.main
        m.step(m.token_state(tokens=list(toks), pos=p, slot=slot))
        m.check()
        return m.argmax()

    def _entry(self, tok, h_rows, pos):
        """one draft-model entry at `pos` on token `tok` and hidden row h_rows [1, 5120] (device); its pick"""
        d = self.draft
        d.set_hidden(h_rows)
        d.step(d.token_state(tokens=int(tok), pos=pos))
        d.check()
        return d.argmax()

    def _drafts(self, seq, p, k, committed):
        """after a main step at p that committed `committed` (= a_0 .. a_k): the draft entries of the committed
        path q = p .. p + k, then K - 1 chained entries; returns the K drafts for the step at p + k + 1"""
        if self.draft_fn is not None:
            return self.draft_fn(seq, p + k + 1, self.K)
        main_x = self.main.x_d
        d1 = None
        for j in range(k + 1):
            d1 = self._entry(committed[j], main_x[j : j + 1], p + j)
        out = [d1]
        q = p + k
        for _ in range(self.K - 1):
            q += 1
            out.append(self._entry(out[-1], self.draft.x_d, q))
        return out

    # ------------------------------------------------------------------------------------------ decode
    def _prompt(self, seq):
        """the prompt through both models, R known tokens per main step (all accepted) and the draft entries of
        every prompt position; returns (p, slot, drafts) for the first decode step at p = len(seq) - 1"""
        P, R = len(seq), self.R
        p = slot = 0
        drafts = [seq[-1]] * self.K
        while p < P - 1:
            n = min(R, P - 1 - p)  # rows with a known next token (positions p .. p + n - 1)
            toks = seq[p : p + n] + [seq[p + n - 1]] * (R - n)
            self._main(toks, p, slot)
            k = n - 1
            drafts = self._drafts(seq, p, k, seq[p + 1 : p + n + 1])
            p, slot = p + n, (slot + k) % R
        return p, slot, drafts

    def generate(self, prompt, n_new):
        """the prompt's tokens then n_new greedy ones, decoded speculatively; returns (tokens, stats)"""
        for m in (self.main, self.draft):
            m.reset()
        seq = [int(t) for t in prompt]
        P = len(seq)
        assert P >= 1
        p, slot, d = self._prompt(seq)
        steps = accepted = 0
        t0 = time.perf_counter()
        while len(seq) < P + n_new:
            a = self._main([seq[p]] + d, p, slot)
            k = 0
            while k < self.K and a[k] == d[k]:
                k += 1
            seq += a[: k + 1]
            d = self._drafts(seq, p, k, a[: k + 1])
            p, slot = p + k + 1, (slot + k) % self.R
            steps += 1
            accepted += k
        total = time.perf_counter() - t0
        return seq[: P + n_new], dict(steps=steps, accepted_drafts=accepted, tokens_per_step=(len(seq) - P) / steps,
                                      ms_per_step=1e3 * total / steps, tok_s=(len(seq) - P) / total)

    # ---- streaming, for the vLLM block adapter (mtp.py:284-346): start() per request, then next_block() per decode
    # step. Host driven: a block runs the steps it needs when it is asked for.

    def start(self, prompt):
        """the prompt through both models and the first verify step: returns that step's row-0 logits [vocab]
        (the first token is their argmax); the other tokens it committed wait for next_block"""
        for m in (self.main, self.draft):
            m.reset()
        seq = [int(t) for t in prompt]
        p, slot, d = self._prompt(seq)
        a = self._main([seq[p]] + d, p, slot)
        logits = self.main.logits()[0].clone()
        k = 0
        while k < self.K and a[k] == d[k]:
            k += 1
        seq += a[: k + 1]
        self._d = self._drafts(seq, p, k, a[: k + 1])
        self._seq, self._p, self._slot = seq, p + k + 1, (slot + k) % self.R
        self._carry = a[1 : k + 1]
        return logits

    def next_block(self, n, limit):
        """the next n committed tokens, or fewer once a step would pass position `limit`"""
        while len(self._carry) < n and self._p + self.R < limit:
            p, slot, d = self._p, self._slot, self._d
            a = self._main([self._seq[p]] + d, p, slot)
            k = 0
            while k < self.K and a[k] == d[k]:
                k += 1
            self._seq += a[: k + 1]
            self._carry += a[: k + 1]
            self._d = self._drafts(self._seq, p, k, a[: k + 1])
            self._p, self._slot = p + k + 1, (slot + k) % self.R
        block, self._carry = self._carry[:n], self._carry[n:]
        return block

    def stop(self):
        """end the request"""
        self._carry, self._seq = [], []

    def greedy(self, prompt, n_new):
        """plain greedy decode on the main model's verify step (every row repeats row 0's token and only row 0 is
        kept): the tokens speculative decode must reproduce"""
        self.main.reset()
        seq = [int(t) for t in prompt]
        p = slot = 0
        while len(seq) < len(prompt) + n_new:
            a = self._main([seq[p]] * self.R, p, slot)
            if p + 1 >= len(seq):
                seq.append(a[0])
            p += 1
        return seq
