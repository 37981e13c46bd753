"""Speculative decoding through the full model (needs a B200): draft ->
verify_tokens over [current, drafts] in every layer -> commit_verified of the
accepted prefix (the rest rolled back), as ``Qwen3SparseModel.speculative_generate``
runs it (reference: ``ModelRunner.run_verify``, model_runner.py:478-507;
``M12LayerRuntime.verify_tokens`` / ``commit_verified`` / ``rollback_verified``,
m12_runtime.py:656-807; proposer interface, sparse/proposers.py).

A random-init target model (6 layers of the Qwen3-4B architecture) over an
8K-token prompt.  The drafts come from a scripted proposer that proposes the
target's own plain greedy decode, verified per query (lossless: each row
attends its own Top-K blocks, as the decode step of that token would; they
are accepted unless the verify pass, whose recent window does not slide inside
the pass, flips a near-tie), from
the n-gram proposer and from a random-init static-graph draft model.  Checked:
every verify call of every layer against the fp32 oracle (its selection modulo
score ties, its output within the parity tolerance) with the oracle committing
the same tokens; the loop's bookkeeping (positions, every layer's history
length); that the emitted tokens follow the target's greedy choice over the
verified rows; and that no kernel reported an error.
"""
import gc

import pytest
import torch

from helpers import orc, pkg
from test_model_tokens import _shadowed_runtime

pytestmark = pytest.mark.gpu
DEV = "cuda"
PROMPT, STEPS, K, LAYERS = 8192 + 200, 32, 4, 6
TIE_BAND = 0.5  # logit units: verify rows and decode steps differ by one old recent token


class EmptyProposer:
    def prefill(self, prompt_ids):
        pass

    def propose(self, last_token, k, pos):
        return []

    def note_accepted(self, tokens):
        pass


class ScriptedProposer(EmptyProposer):
    """Proposes the continuation of a known token sequence S by position (S[0]
    is the token at position P, the prompt length), whether or not the loop
    still follows S."""

    def __init__(self, seq, prompt_len):
        self.seq, self.P = list(seq), prompt_len

    def propose(self, last_token, k, pos):
        i = pos - self.P
        return self.seq[i + 1:i + 1 + k] if 0 <= i < len(self.seq) else []


def _model(H, nkv, make=None, seed=7):
    arch = H.Qwen3Arch(num_layers=LAYERS)
    mk = make or (lambda i: nkv.M12LayerRuntime(i, nkv.M12Config(max_model_len=PROMPT + 2048, device=DEV)))
    return H.Qwen3SparseModel(arch, mk, device=DEV, seed=seed)


def _prompt(vocab):
    return torch.randint(0, vocab, (PROMPT,), generator=torch.Generator().manual_seed(11))


def _check_state(model, toks):
    assert model.position == PROMPT + len(toks) - 1
    for rt in model.runtimes:
        assert rt.valid_len == model.position
        assert int(rt._att_ws[:4].view(torch.int32).item()) == 0
    model.check_errors()


def test_speculative_loop_follows_greedy_and_matches_oracle():
    nkv = pkg()
    from importlib import import_module
    H = import_module(nkv.__name__ + ".qwen3_harness")
    prompt = _prompt(H.Qwen3Arch().vocab_size)
    # plain greedy decode (rounds without drafts are decode steps)
    A = _model(H, nkv)
    s0, st0 = A.speculative_generate(prompt, STEPS, EmptyProposer())
    assert st0["verify_rounds"] == 0 and len(s0) == STEPS + 1
    _check_state(A, s0)
    del A
    gc.collect()
    torch.cuda.empty_cache()

    # scripted drafts, every layer shadowed by the oracle
    Shadowed = _shadowed_runtime(nkv)
    failures, logs = [], []
    ocfg = orc.OracleConfig(device=DEV)

    def make(i):
        rt = Shadowed(i, nkv.M12Config(max_model_len=PROMPT + 2048, device=DEV))
        logs.append([])
        rt.setup(ocfg, failures, logs[-1])
        return rt
    B = _model(H, nkv, make)
    rows = []
    verify = B.verify

    def verify_logged(tokens):
        logits = verify(tokens)
        rows.append((list(tokens), logits.float().cpu()))
        return logits
    B.verify = verify_logged
    s1, st1 = B.speculative_generate(prompt, STEPS, ScriptedProposer(s0, PROMPT), k=K, lossless=True)
    assert not failures, f"{len(failures)} calls outside the parity bounds: {failures[:6]}"
    assert st1["verify_rounds"] >= 1 and st1["proposed"] >= K
    assert all(sum(w == "verify" for w, _ in lg) == st1["verify_rounds"] for lg in logs)
    _check_state(B, s1)
    # every emitted token is the target's greedy choice over the verified rows:
    # accepted drafts equal the argmax of the row before them, the last token
    # of a round is the argmax of the row after the accepted prefix
    i = 1
    for tokens, logits in rows:
        tgt = logits.argmax(dim=-1).tolist()
        while i < len(s1) and s1[i - 1] != tokens[0]:
            i += 1  # decode-step rounds between verify rounds
        n = 0
        while n + 1 < len(tokens) and tokens[n + 1] == tgt[n]:
            n += 1
        assert s1[i:i + n + 1] == tgt[:n + 1][:len(s1) - i], (tokens, tgt, s1[i:i + n + 1])
        i += n + 1
    # while the loop follows the plain greedy decode, its drafts are accepted
    # except where a verify row's top-2 logits are a near-tie (the first round
    # starts on it; after a rejection the two runs part)
    tokens, logits = rows[0]
    assert tokens == s0[:len(tokens)]
    tgt = logits.argmax(dim=-1).tolist()
    gap = None
    for j in range(1, len(tokens)):
        if tokens[j] != tgt[j - 1]:
            gap = float(logits[j - 1, tgt[j - 1]] - logits[j - 1, tokens[j]])
            break
    print(f"\nscripted drafts: {st1['accepted']}/{st1['proposed']} accepted in {st1['verify_rounds']} verify "
          f"rounds; first round's rejection logit gap {gap}")
    assert gap is None or gap < TIE_BAND, gap


@pytest.mark.parametrize("which", ["ngram", "draft_model", "draft_model_lossless"])
def test_speculative_loop_with_proposers(which):
    nkv = pkg()
    from importlib import import_module
    H = import_module(nkv.__name__ + ".qwen3_harness")
    P = import_module(nkv.__name__ + ".proposers")
    arch = H.Qwen3Arch()
    # a prompt that repeats a pattern, so that the n-gram proposer has matches
    g = torch.Generator().manual_seed(12)
    pat = torch.randint(0, arch.vocab_size, (97,), generator=g)
    prompt = pat.repeat(PROMPT // 97 + 1)[:PROMPT].clone()
    model = _model(H, nkv)
    if which.startswith("draft_model"):
        proposer = P.DraftModelProposer(P.StaticDraftModel(P.DraftArch(num_layers=2), window=1024, device=DEV))
    else:
        proposer = P.NgramProposer(n=1, max_k=K)
    toks, st = model.speculative_generate(prompt, 24, proposer, k=K, lossless=which.endswith("lossless"))
    print(f"\n{which}: {st}")
    assert len(toks) == 25
    if which.startswith("draft_model"):  # a draft model proposes in every round but a last one-token round
        assert st["verify_rounds"] >= st["rounds"] - 1 and st["proposed"] >= K * (st["rounds"] - K - 1)
    _check_state(model, toks)
