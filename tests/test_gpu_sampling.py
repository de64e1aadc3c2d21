"""Device-resident acceptance and sampling (csrc/sampling.cu) against the
reference's sampling functions and decoder.

* every function on every seeded case of tests/sampling_cases.py: sampled
  indices, first rejections and round outcomes equal the reference's
  (tests/golden/sampling.json); acceptance probabilities within 2 ulp of
  the reference's extended-precision values; residual and normalised rows
  within 1e-15 of the oracle's (which equals the reference's bit for bit);
* the fused verification round, one sequence and batched, with ragged
  proposal counts, without bonus, on float32 and on unnormalised rows;
* the reference tests' known answers and error cases through
  DeviceSamplingBackend (tests/test_native.py:40-90 of the reference);
* whole decodes: the reference's own SpeculativeDecoder (src/specdecode/
  decoder.py, unchanged, from the copy of its package in oracle/_ref/) with
  DeviceSamplingBackend as its sampling backend gives the recorded tokens,
  events, statistics and generator state, also when the target model scores
  a whole proposal in one call (score_proposal);
* a 64-sequence, 128 256-token-vocabulary round checked by properties that
  hold at any size.
"""

from __future__ import annotations

import hashlib
import json
import random
from pathlib import Path

import numpy as np
import pytest

import sampling_cases as sc

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "sampling.json").read_text())
CASES = {c.name: c for c in sc.cases()}


def _t(device, a, dtype=None):
    import torch

    return torch.as_tensor(np.asarray(a), dtype=dtype or torch.float64, device=device)


def within_ulps(got, want, ulps=2):
    got, want = np.asarray(got, dtype=np.float64), np.asarray(want, dtype=np.float64)
    scale = np.spacing(np.maximum(np.abs(got), np.abs(want)))
    return bool(np.all(np.abs(got - want) <= ulps * scale))


def _normalised(case):
    from oracle import sampling as orc

    tn = np.array([orc.python_normalize(r) for r in case.target])
    dn = np.array([orc.python_normalize(r) for r in case.draft])
    return tn, dn


@pytest.mark.parametrize("record", GOLDEN["cases"], ids=lambda r: r["name"])
def test_functions_match_the_reference(device, record):
    import torch

    from oracle import sampling as orc
    from specdecode_b200 import sampling as smp

    case = CASES[record["name"]]
    n = len(case.proposed)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    t, d = _t(device, case.target), _t(device, case.draft)
    acc = smp.acceptance_rows(t[:n], d, _t(device, case.proposed, torch.int64), status=status)
    assert within_ulps(acc.cpu().numpy(), record["acceptance"]), (acc.tolist(), record["acceptance"])
    rej = smp.first_rejection_rows(_t(device, [record["acceptance"]]), _t(device, [case.uniforms[:n]]), status=status)
    assert int(rej.item()) == record["first_rejection"]
    # every target row at every draw of the case
    R = n + 1
    weights = t.repeat_interleave(R, dim=0)
    uniforms = _t(device, case.uniforms * R)
    samples = smp.sample_rows(weights, uniforms, status=status).view(R, R).tolist()
    assert samples == record["categorical"]
    res = smp.residual_rows(t[:n], d, status=status).cpu().numpy()
    want = np.array([orc.residual_weights(case.target[i], case.draft[i]) for i in range(n)])
    assert np.abs(res - want).max() <= 1e-15
    norm = smp.normalize_rows(t, status=status).cpu().numpy()
    want = np.array([orc.normalize(r) for r in case.target])
    assert within_ulps(norm, want, 1)
    assert int(status.item()) == 0


def _round_inputs(device, case, normalised=True, dtype=None):
    import torch

    tn, dn = _normalised(case) if normalised else (case.target, case.draft)
    return (_t(device, tn[None], dtype), _t(device, dn[None], dtype), _t(device, [case.proposed], torch.int64),
            _t(device, [case.uniforms]))


@pytest.mark.parametrize("record", GOLDEN["cases"], ids=lambda r: r["name"])
def test_verify_round_matches_the_reference_decoder(device, record):
    import torch

    from specdecode_b200.sampling import verify_batch

    case = CASES[record["name"]]
    want = record["round"]
    bonus = _t(device, [1 if case.bonus else 0], torch.uint8)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    variants = [dict(normalised=True), dict(normalised=False)]
    if case.name.startswith(("softmax", "near", "identical", "v1")):
        variants.append(dict(normalised=False, dtype=torch.float32))  # rows exact in float32
    for v, reuse in [(v, r) for v in variants for r in (True, False)]:
        t, d, tok, u = _round_inputs(device, case, **v)
        acc, token, probs = verify_batch(t, d, tok, u, bonus_allowed=bonus, status=status, reuse_row_sums=reuse)
        assert (int(acc.item()), int(token.item())) == (want["accepted"], want["token"]), v
        if v["normalised"]:
            assert within_ulps(probs[0].cpu().numpy(), want["probabilities"]), v
    assert int(status.item()) == 0


def test_verify_batched_with_ragged_windows(device):
    """The eight near-draft cases as one batch, with windows cut to 6..1
    proposals and two sequences without bonus; expected rounds from the
    oracle, which reproduces the reference bit for bit."""
    import torch

    from oracle import sampling as orc
    from specdecode_b200.sampling import verify_batch

    names = [f"near_v500_s{s}" for s in range(30, 38)]
    cases = [CASES[n] for n in names]
    counts = [6, 5, 4, 3, 2, 1, 6, 6]
    bonus = [1, 1, 1, 1, 1, 1, 0, 0]
    tn = np.stack([_normalised(c)[0] for c in cases])
    dn = np.stack([_normalised(c)[1] for c in cases])
    tok = np.array([c.proposed for c in cases])
    uni = np.array([c.uniforms for c in cases])
    target = tn  # a window cut to n proposals takes its bonus from target row n
    status = torch.zeros(1, dtype=torch.int32, device=device)
    acc, token, probs = verify_batch(_t(device, target), _t(device, dn), _t(device, tok, torch.int64),
                                     _t(device, uni), proposal_counts=_t(device, counts, torch.int64),
                                     bonus_allowed=_t(device, bonus, torch.uint8), status=status)
    assert int(status.item()) == 0
    for s, (case, n) in enumerate(zip(cases, counts)):
        want = orc.verify_round([tuple(r) for r in target[s, : n + 1]], [tuple(r) for r in dn[s, :n]],
                                case.proposed[:n], case.uniforms, bool(bonus[s]))
        assert (int(acc[s]), int(token[s])) == (want.accepted, want.token), case.name
        assert within_ulps(probs[s, :n].cpu().numpy(), want.probabilities)


def test_sample_never_lands_on_trailing_zero_weights(device):
    """Rows whose positive weights end early in a long row (zeros after
    them, across whole chunks of the kernel): a uniform just below 1 takes
    the last positive weight, as the reference's running sum does, never a
    zero-weight index after it."""
    import torch

    from specdecode_b200.sampling import sample_rows

    vocab = 3000
    rows = []
    for last in (1, 127, 128, 129, 1000, 2047):
        w = np.zeros(vocab)
        w[: last + 1] = np.linspace(1.0, 2.0, last + 1)
        rows.append(w)
    weights = torch.tensor(np.array(rows), device=device)
    uniforms = torch.full((len(rows),), 1.0 - 2.0 ** -53, dtype=torch.float64, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    got = sample_rows(weights, uniforms, status=status).cpu().tolist()
    assert int(status.item()) == 0
    assert got == [1, 127, 128, 129, 1000, 2047]


def test_device_backend_known_answers(device):
    from specdecode_b200.sampling import DeviceSamplingBackend

    kat = GOLDEN["kat"]
    backend = DeviceSamplingBackend(device)
    w = sc.KAT_CATEGORICAL_WEIGHTS
    assert np.allclose(backend.normalize(w), kat["normalized"], rtol=0, atol=1e-12)
    assert [backend.categorical(w, u) for u in sc.KAT_CATEGORICAL_UNIFORMS] == kat["categorical"]
    assert within_ulps(backend.acceptance_probabilities(sc.KAT_TARGET_ROWS, sc.KAT_DRAFT_ROWS, sc.KAT_TOKENS),
                       kat["acceptance"])
    assert np.allclose(backend.residual_weights(sc.KAT_TARGET_ROWS[0], sc.KAT_DRAFT_ROWS[0]), kat["residual_0"],
                       rtol=0, atol=1e-15)
    assert np.allclose(backend.residual_weights(sc.KAT_TARGET_ROWS[2], sc.KAT_TARGET_ROWS[2]),
                       kat["residual_same"], rtol=0, atol=1e-15)
    result = backend.first_rejection(sc.KAT_REJECTION_PROBABILITIES, sc.KAT_REJECTION_UNIFORMS)
    assert (result.accepted_count, result.rejection_index) == (kat["first_rejection"], kat["first_rejection"])
    result = backend.first_rejection((0.5, 1.0), (0.1, 0.9))
    assert (result.accepted_count, result.rejection_index) == (2, None)


@pytest.mark.parametrize("call,status", [
    (lambda b: b.categorical((0.5, -0.5), 0.1), 4),
    (lambda b: b.categorical((0.5, 0.5), 1.0), 7),
    (lambda b: b.categorical((0.0, 0.0), 0.1), 5),
    (lambda b: b.categorical((float("nan"), 1.0), 0.1), 3),
    (lambda b: b.acceptance_probabilities(((1.0, 0.0),), ((1.0, 0.0),), (2,)), 6),
    (lambda b: b.residual_weights((0.0, 0.0), (1.0, 0.0)), 5),
    (lambda b: b.first_rejection((1.5,), (0.1,)), 4),
    (lambda b: b.first_rejection((0.5,), (-0.1,)), 7),
    (lambda b: b.residual_weights((0.5, 0.5), (1.0,)), None),
    (lambda b: b.acceptance_probabilities(((1.0, 0.0),), (), (0,)), None),
])
def test_device_backend_errors_are_not_hidden(device, call, status):
    """The reference's validation cases (tests/test_native.py:84-90) and the
    statuses its library returns for them (oracle tests pin those)."""
    from specdecode_b200 import NativeBackendError
    from specdecode_b200.sampling import DeviceSamplingBackend

    backend = DeviceSamplingBackend(device)
    with pytest.raises(NativeBackendError) as err:
        call(backend)
    if status is not None:
        assert err.value.status == status
    # the backend stays usable after a device-side fault
    assert backend.categorical((1.0, 3.0), 0.5) == 1


def test_faulted_sequences_are_marked_and_others_decided(device):
    import torch

    from specdecode_b200 import _lib
    from specdecode_b200.sampling import verify_batch

    case = CASES["near_v500_s30"]
    tn, dn = _normalised(case)
    S = 5
    target = np.repeat(tn[None], S, axis=0)
    draft = np.repeat(dn[None], S, axis=0)
    tok = np.repeat(np.array([case.proposed]), S, axis=0)
    uni = np.repeat(np.array([case.uniforms]), S, axis=0)
    target[1, 2, 7] = -1.0  # negative weight
    tok[2, 0] = 500  # outside the vocabulary
    uni[3, 0] = 1.0  # not in [0, 1)
    counts = [6, 6, 6, 6, 0]  # 0 proposals: not a round
    status = torch.zeros(1, dtype=torch.int32, device=device)
    acc, token, _ = verify_batch(_t(device, target), _t(device, draft), _t(device, tok, torch.int64),
                                 _t(device, uni), proposal_counts=_t(device, counts, torch.int64), status=status)
    bits = int(status.item())
    for bit in (_lib.FAULT_NEGATIVE_WEIGHT, _lib.FAULT_TOKEN_RANGE, _lib.FAULT_INVALID_UNIFORM,
                _lib.FAULT_PROPOSAL_COUNT):
        assert bits & bit, hex(bits)
    assert acc[1:].tolist() == [-1, -1, -1, -1] and token[1:].tolist() == [-1, -1, -1, -1]
    want = GOLDEN["cases"][[r["name"] for r in GOLDEN["cases"]].index(case.name)]["round"]
    assert (int(acc[0]), int(token[0])) == (want["accepted"], want["token"])


def _reference_decoder():
    """The reference's decoder, config and table model from oracle/_ref/."""
    from oracle.reference_runs import ReferenceUnavailable, reference_package

    try:
        reference_package()
    except ReferenceUnavailable as error:
        pytest.skip(str(error))
    from specdecode.config import DecodeConfig
    from specdecode.decoder import SpeculativeDecoder
    from specdecode.models import TableModel

    return DecodeConfig, SpeculativeDecoder, TableModel


def _check_decode(result, events, rng, record):
    assert list(result.generated_tokens) == record["generated"]
    assert [e.source for e in events] == record["sources"]
    assert [e.index for e in events] == record["indices"]
    s = result.stats
    assert dict(drafted_tokens=s.drafted_tokens, accepted_tokens=s.accepted_tokens,
                rejected_tokens=s.rejected_tokens, target_tokens=s.target_tokens,
                verification_rounds=s.verification_rounds, fallback_steps=s.fallback_steps) == record["stats"]
    assert hashlib.sha256(repr(rng.getstate()).encode()).hexdigest() == record["rng_sha"]


@pytest.mark.parametrize("scoring", [False, True], ids=["next_token_probs", "score_proposal"])
@pytest.mark.parametrize("record", GOLDEN["decodes"], ids=lambda r: r["name"])
def test_reference_decoder_on_the_device_backend(device, record, scoring):
    """The reference's SpeculativeDecoder, unchanged, drives the device
    kernels through DeviceSamplingBackend and reproduces its recorded run
    (made with its own native and Python backends, tests/test_native.py:92-124
    of the reference).  With ``score_proposal`` the target's rows for a whole
    proposal come from one call (src/specdecode/decoder.py:113-136), the path
    the reference's Hugging Face adapter takes."""
    from specdecode_b200.sampling import DeviceSamplingBackend

    DecodeConfig, SpeculativeDecoder, TableModel = _reference_decoder()

    class ScoringTable(TableModel):
        calls = 0

        def score_proposal(self, prefix, proposed):
            ScoringTable.calls += 1
            return [self.next_token_probs(list(prefix) + list(proposed[:i])) for i in range(len(proposed) + 1)]

    run = next(r for r in sc.decode_runs() if r["name"] == record["name"])
    (dt, dd), (tt, td) = sc.tables_for(run)
    config = DecodeConfig(max_new_tokens=run["max_new_tokens"], eos_token_id=run["eos_token_id"],
                          initial_draft_tokens=run.get("initial_draft_tokens", 4),
                          dynamic_draft=run.get("dynamic_draft", True))
    target = (ScoringTable if scoring else TableModel)(tt, td)
    rng = random.Random(run["seed"])
    events = []
    decoder = SpeculativeDecoder(TableModel(dt, dd), target, config, rng=rng,
                                 sampling_backend=DeviceSamplingBackend(device))
    result = decoder.generate(run["prompt"], on_token=events.append)
    _check_decode(result, events, rng, record)
    if scoring:
        assert ScoringTable.calls == result.stats.verification_rounds > 0


def test_large_vocabulary_round_properties(device):
    """64 sequences, 6 proposals, 128 256 tokens, float32 softmax rows: each
    decision is checked against float64 sums, whose error at this size stays
    below 1e-10 of the total, so a sample outside that band is a bug."""
    import torch

    from specdecode_b200.sampling import verify_batch

    S, k, V = 64, 6, 128256
    g = torch.Generator(device=device).manual_seed(5)
    logits = torch.randn((S, k + 1, V), generator=g, device=device) * 2.0
    target = torch.softmax(logits, dim=-1)
    draft = torch.softmax(logits[:, :k] + 0.5 * torch.randn((S, k, V), generator=g, device=device), dim=-1)
    tok = torch.multinomial(draft.reshape(-1, V), 1, generator=g).view(S, k)
    uni = torch.rand((S, k + 1), generator=g, device=device, dtype=torch.float64)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    acc, token, probs = verify_batch(target, draft, tok, uni, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    t64, d64 = target.double(), draft.double()
    st, sd = t64.sum(-1), d64.sum(-1)
    p = t64[:, :k].gather(2, tok[..., None]).squeeze(2) / st[:, :k]
    q = d64.gather(2, tok[..., None]).squeeze(2) / sd
    want = torch.where(q > 0, torch.clamp(p / q, max=1.0), torch.ones_like(p))
    assert torch.allclose(probs, want, rtol=1e-12, atol=0)
    rejected = accepted = 0
    for s in range(S):
        j = int(acc[s])
        a = probs[s].tolist()
        u = uni[s].tolist()
        assert all(u[i] < a[i] for i in range(j))
        if j < k:
            assert not u[j] < a[j]
            w = torch.clamp(t64[s, j] / st[s, j] - d64[s, j] / sd[s, j], min=0.0)
            thr = u[j + 1] * float(w.sum())
            rejected += 1
        else:
            w = t64[s, k]
            thr = u[k] * float(w.sum())
            accepted += 1
        c = int(token[s])
        cum = torch.cumsum(w, 0)
        tol = 1e-10 * float(cum[-1])  # float64 running sums over 128 256 terms
        assert float(w[c]) > 0.0
        before = float(cum[c - 1]) if c > 0 else 0.0
        assert before <= thr + tol and thr < float(cum[c]) + tol, (s, c, before, thr)
    assert rejected > 0 and accepted > 0


def test_host_inputs_and_wrong_outputs_are_refused_or_moved(device):
    """Rows on the host, an output buffer or status word of the wrong kind
    raise before a launch; small per-row inputs on the host are copied to the
    rows' device."""
    import torch

    from specdecode_b200.sampling import sample_rows, verify_batch

    w = torch.tensor([[0.2, 0.3, 0.5], [1.0, 0.0, 0.0]], dtype=torch.float64)
    with pytest.raises(ValueError):
        sample_rows(w, torch.tensor([0.5, 0.5], dtype=torch.float64))
    wd = w.to(device)
    got = sample_rows(wd, torch.tensor([0.6, 0.9], dtype=torch.float64))  # uniforms on the host
    assert got.cpu().tolist() == [2, 0]
    with pytest.raises(ValueError):
        sample_rows(wd, torch.tensor([0.6, 0.9]), out=torch.empty(3, dtype=torch.int64, device=device))
    with pytest.raises(ValueError):
        sample_rows(wd, torch.tensor([0.6, 0.9]), status=torch.zeros(1, dtype=torch.int32))
    target = torch.full((1, 2, 4), 0.25, dtype=torch.float64, device=device)
    draft = torch.full((1, 1, 4), 0.25, dtype=torch.float64, device=device)
    acc, tok, _ = verify_batch(target, draft, torch.tensor([[1]]), torch.tensor([[0.5, 0.1]], dtype=torch.float64))
    assert acc.cpu().tolist() == [1] and 0 <= int(tok.item()) < 4
    with pytest.raises(ValueError):
        verify_batch(target, draft, torch.tensor([[1]]), torch.tensor([[0.5, 0.1]], dtype=torch.float64),
                     out_accepted=torch.empty(2, dtype=torch.int64, device=device))
