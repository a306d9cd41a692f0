"""GPU: the speculative verify/rollback loop of lisa-rs driven end to end
through the C ABI with a fake drafter.

lisa-rs decodes with MTP speculation: `run_block3_loop`
(src/speculative/mod.rs:102-198) verifies [bonus, d0, d1] in one M=3
attention call (`verify_block3_decode_device`), accepts the drafts greedily
(`accept_greedy`, mod.rs:16-32), keeps the accepted prefix of the KV cache
(`commit_verified_prefix`) and continues from the last emitted token. Greedy
speculation is exact only if a verify row equals the same row decoded alone,
bit for bit — the M=1 / M=3 identity this library guarantees.

Here the target model is one attention layer of this library plus a toy
token embedding (seeded q_proj/k_proj/v_proj outputs per token id) and a toy
output head (argmax of a fixed random projection of the gated output). The
drafter is fake: it proposes the true next token with probability 0.6 and a
random token otherwise, so accepts, partial accepts and full rejections all
occur. The loop must emit exactly the tokens of plain M=1 greedy decoding and
leave the same KV cache.
"""
import numpy as np
import pytest

from helpers import KROW, OROW, QROW, norm_weights

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import weights  # noqa: E402

VOCAB = 48
PROMPT = 40
MAX_TOKENS = 30


class ToyTarget:
    """One attention layer behind a toy embedding and output head."""

    def __init__(self, seed: int, capacity: int):
        rng = np.random.default_rng(seed)
        self.eq = torch.from_numpy(rng.standard_normal((VOCAB, QROW)).astype(np.float32)).cuda()
        self.ek = torch.from_numpy(rng.standard_normal((VOCAB, KROW)).astype(np.float32)).cuda()
        self.ev = torch.from_numpy(rng.standard_normal((VOCAB, KROW)).astype(np.float32)).cuda()
        self.head = torch.from_numpy(rng.standard_normal((VOCAB, OROW))).cuda()  # f64
        qn, kn = norm_weights(rng)
        self.w = weights(qn, kn)
        self.runner = lisa_attn.AttnRunner(1, capacity)

    def inputs(self, tokens):
        idx = torch.tensor(tokens, dtype=torch.long, device="cuda")
        return self.eq[idx].contiguous(), self.ek[idx].contiguous(), self.ev[idx].contiguous()

    def next_tokens(self, out):
        """Greedy next token of each output row (ties: lowest id)."""
        logits = out.double() @ self.head.t()
        return [int(t) for t in torch.argmax(logits, dim=1).tolist()]

    def prefill(self, tokens):
        out = self.runner.forward_prefill(0, *self.inputs(tokens), self.w)
        self.runner.advance(len(tokens))
        return self.next_tokens(out[-1:])[0]

    def forward_token_decode(self, token):
        out = self.runner.forward_decode(0, *self.inputs([token]), self.w)
        self.runner.advance(1)
        return self.next_tokens(out)[0]

    def verify_block3(self, tokens):
        out = self.runner.verify_block3(0, *self.inputs(tokens), self.w)
        self.runner.advance(3, verify=True)
        return self.next_tokens(out)


def accept_greedy(drafts, target_tokens):
    """speculative/mod.rs:16-32."""
    assert len(target_tokens) == len(drafts) + 1
    accepted = 0
    while accepted < len(drafts) and drafts[accepted] == target_tokens[accepted]:
        accepted += 1
    return accepted, list(drafts[:accepted]) + [target_tokens[accepted]]


def greedy_sequential(model, bonus, max_tokens):
    tokens = []
    while len(tokens) < max_tokens:
        bonus = model.forward_token_decode(bonus)
        tokens.append(bonus)
    return tokens


def greedy_block3(model, bonus, max_tokens, drafter):
    """run_block3_loop (speculative/mod.rs:102-198) without the MTP drafter's
    own cache: drafts come from `drafter(emitted_so_far)`."""
    tokens, rounds, accepted_total = [], 0, 0
    while len(tokens) < max_tokens:
        remaining = max_tokens - len(tokens)
        if remaining < 3:
            for _ in range(remaining):
                bonus = model.forward_token_decode(bonus)
                tokens.append(bonus)
            break
        d = drafter(len(tokens))
        target = model.verify_block3([bonus, d[0], d[1]])
        accepted, emitted = accept_greedy(d, target)
        model.runner.commit_verified_prefix(accepted + 1)
        bonus = emitted[-1]
        tokens.extend(emitted)
        rounds += 1
        accepted_total += accepted
    return tokens, rounds, accepted_total


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_block3_loop_equals_sequential_greedy(seed):
    cap = PROMPT + MAX_TOKENS + 8
    rng = np.random.default_rng(9000 + seed)
    prompt = rng.integers(0, VOCAB, size=PROMPT).tolist()

    seq = ToyTarget(seed, cap)
    bonus0 = seq.prefill(prompt)
    want = greedy_sequential(seq, bonus0, MAX_TOKENS)

    spec = ToyTarget(seed, cap)
    assert spec.prefill(prompt) == bonus0
    draft_rng = np.random.default_rng(500 + seed)

    def drafter(n_emitted):
        out = []
        for i in range(2):
            truth = want[n_emitted + i] if n_emitted + i < len(want) else 0
            out.append(truth if draft_rng.random() < 0.6 else int(draft_rng.integers(0, VOCAB)))
        return out

    got, rounds, accepted = greedy_block3(spec, bonus0, MAX_TOKENS, drafter)
    assert got == want
    assert rounds > 0 and 0 < accepted < 2 * rounds  # both accepted and rejected drafts occurred
    # the committed KV prefix is the sequential one, bit for bit
    n = PROMPT + MAX_TOKENS
    assert spec.runner.position() == seq.runner.position() == n
    for a, b in zip(spec.runner.kv_cache(0), seq.runner.kv_cache(0)):
        assert torch.equal(a[:, :n], b[:, :n])


def mtp_reconcile_plan(draft_count, round_appended, accepted):
    """speculative/mod.rs:49-65: keep the drafts already appended this round
    that were accepted, replay the accepted ones not in the cache, then the
    replacement / bonus token."""
    assert accepted <= draft_count and round_appended <= draft_count
    keep = min(accepted, round_appended)
    replay = [("draft", i) for i in range(keep, accepted)] + [("replacement", None)]
    return round_appended - keep, replay


class ToyDrafter(ToyTarget):
    """The MTP drafter's attention: a 1-layer context of its own (own toy
    embedding), advanced one position per forward and trimmed by the
    reconcile plan; `tokens` is the token sequence its live KV prefix must
    hold."""

    def __init__(self, seed, capacity):
        super().__init__(seed + 777, capacity)
        self.tokens = []

    def forward(self, token):
        out = self.runner.forward_decode(0, *self.inputs([token]), self.w)
        self.runner.advance(1)
        self.tokens.append(token)
        return self.next_tokens(out)[0]

    def trim_state(self, n):
        self.runner.trim_state(n)
        del self.tokens[len(self.tokens) - n:]


@pytest.mark.parametrize("seed", [4, 5])
def test_block3_loop_with_a_drafter_context(seed):
    """run_block3_loop (speculative/mod.rs:102-198) with the drafter side too:
    the drafter appends its forwards to its own 1-layer context, and after
    every verify applies mtp_reconcile_plan + trim_state (mod.rs:167) and
    replays the plan's last entry. The emitted tokens equal sequential greedy
    decoding, and the drafter's live KV prefix equals a fresh drafter that
    decoded the same token sequence one position at a time."""
    cap = PROMPT + 2 * MAX_TOKENS + 16
    rng = np.random.default_rng(9100 + seed)
    prompt = rng.integers(0, VOCAB, size=PROMPT).tolist()
    seq = ToyTarget(seed, cap)
    bonus = seq.prefill(prompt)
    want = greedy_sequential(seq, bonus, MAX_TOKENS)

    spec = ToyTarget(seed, cap)
    assert spec.prefill(prompt) == bonus
    mtp = ToyDrafter(seed, cap)
    mix = np.random.default_rng(600 + seed)

    def draft(own, n_emitted):
        truth = want[n_emitted] if n_emitted < len(want) else 0
        return truth if mix.random() < 0.6 else own

    tokens, seed_tok, rounds, trims = [], None, 0, 0
    while len(tokens) < MAX_TOKENS:
        remaining = MAX_TOKENS - len(tokens)
        if remaining < 3:
            for _ in range(remaining):
                bonus = spec.forward_token_decode(bonus)
                tokens.append(bonus)
            break
        if seed_tok is not None:
            d0 = seed_tok
            d1 = draft(mtp.forward(d0), len(tokens) + 1)
            round_appended = 1
        else:
            d0 = draft(mtp.forward(bonus), len(tokens))
            d1 = draft(mtp.forward(d0), len(tokens) + 1)
            round_appended = 2
        drafts = [d0, d1]
        target = spec.verify_block3([bonus, d0, d1])
        accepted, emitted = accept_greedy(drafts, target)
        spec.runner.commit_verified_prefix(accepted + 1)
        trim, replay = mtp_reconcile_plan(2, round_appended, accepted)
        mtp.trim_state(trim)
        trims += trim
        kind, index = replay[-1]
        token = drafts[index] if kind == "draft" else emitted[-1]
        seed_tok = draft(mtp.forward(token), len(tokens) + len(emitted))
        bonus = emitted[-1]
        tokens.extend(emitted)
        rounds += 1
    assert tokens == want
    assert rounds > 0 and trims > 0
    # the drafter's live prefix: same rows as a fresh drafter fed mtp.tokens one by one
    fresh = ToyDrafter(seed, cap)
    for t in mtp.tokens:
        fresh.forward(t)
    n = len(mtp.tokens)
    assert mtp.runner.position() == fresh.runner.position() == n
    for a, b in zip(mtp.runner.kv_cache(0), fresh.runner.kv_cache(0)):
        assert torch.equal(a[:, :n], b[:, :n])
