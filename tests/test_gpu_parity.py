"""GPU parity: the B200 kernels against the reference's own outputs (golden
fixtures) and against the CPU oracle, through the C ABI and through the
drop-in Python API. Bit-exact: tokens, accepted_len and status must be equal.

Cases restate the reference's suites (tests/test_cuda.py, tests/test_fused.py,
tests/edge, tests/invariance) and the benchmark configurations at full size.
"""
import dataclasses

import numpy as np
import pytest

import oracle
import workloads
from tests import cases as C
from tests import golden_io
from tests.gpu_helpers import assert_same, device_inputs, run_abi, run_api

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from exactsample_b200.cuda import load_library
    load_library()


SMALL = golden_io.small()


@pytest.mark.parametrize("list_max", [256, 0])
@pytest.mark.parametrize("entry", SMALL, ids=lambda e: e[0]["name"])
def test_small_golden_through_abi(entry, list_max):
    case, expected = entry
    got = run_abi(device_inputs(case), mode=case["mode"], list_max=list_max)
    assert_same(got, expected, context=case["name"])
    assert (got[3] == 1).all()


@pytest.mark.parametrize("entry", SMALL, ids=lambda e: e[0]["name"])
def test_small_golden_reference_dispatch(entry):
    case, expected = entry
    out, _ = run_api(case, dispatch="reference")
    got = (out.tokens.cpu().numpy(), out.accepted_len.cpu().numpy(), out.status.cpu().numpy())
    assert_same(got, expected, context=case["name"])
    assert (out.path_used.cpu().numpy() == 0).all()


@pytest.mark.parametrize("entry", [e for e in SMALL if e[0]["name"].startswith(("dtype_", "mask_", "random_1", "random_3"))],
                         ids=lambda e: e[0]["name"])
def test_strided_inputs_through_api(entry):
    case, expected = entry
    out, work = run_api(case, strided=True)
    got = (out.tokens.cpu().numpy(), out.accepted_len.cpu().numpy(), out.status.cpu().numpy())
    assert_same(got, expected, context=case["name"])


def _large():
    try:
        return golden_io.large_entries()
    except FileNotFoundError:
        return []


@pytest.mark.parametrize("list_max", [256, 0])
@pytest.mark.parametrize("entry", _large(), ids=lambda e: e[0])
def test_large_golden(entry, list_max):
    name, subset, digest, expected = entry
    case = golden_io.large_case(name, subset, digest)
    got = run_abi(device_inputs(case), mode=case["mode"], list_max=list_max)
    assert_same(got, expected, context=name)


def oracle_outputs(case, **kw):
    out = oracle.verify_reference(**C.oracle_inputs(case, oracle), **kw)
    return out.tokens, out.accepted_len, out.status


@pytest.mark.parametrize("name", ["C1", "C2a", "C2b", "C3a", "C3b", "C3b_ratio_full", "C3b_coupled_onehot", "C4"])
def test_benchmark_configuration_full_size(name):
    case = C.workload_case(name)
    expected = oracle_outputs(case)
    for list_max in [256, 0]:
        got = run_abi(device_inputs(case), mode=case["mode"], list_max=list_max)
        assert_same(got, expected, context=f"{name} list_max={list_max}")
    if name == "C3b":
        assert (expected[2] == 2).all()  # coupled mode with full proposals is invalid by contract


@pytest.mark.parametrize("name", ["C1", "C2a", "C2b", "C3a", "C3b_ratio_full", "C3b_coupled_onehot", "C4"])
def test_reference_dispatch_full_size(name):
    """dispatch="reference" runs the independent FP64 kernel (one block per
    row); it must agree with the oracle at full vocabulary, and so with the
    fused kernel."""
    case = C.workload_case(name)
    expected = oracle_outputs(case)
    got = run_abi(device_inputs(case, reference=True), mode=case["mode"], dispatch="reference")
    assert_same(got, expected, context=f"{name} reference dispatch")
    assert (got[3][:len(expected[2])] == 0).all()  # path_used: reference


@pytest.mark.parametrize("setting", ["qwen", "temperature", "top_p"])
def test_sampler_grid_settings(setting):
    """The three settings of the reference's sampler benchmark grid
    (bench/sampler.py:36-41) on bf16 rows: sampling rows, and ratio
    verification whose draft rows need the kept set's mass (temperature
    only: bounds on it settle most tests; top-p only: a list of the largest
    tokens settles the nucleus), against the oracle."""
    import bench
    chosen = bench.SAMPLER_SETTINGS[setting]
    for w in [workloads.sampling(8, chosen, master_seed=61), workloads.verification(6, 4, chosen, master_seed=62)]:
        case = dict(name=f"{setting}_{w.name}", logits=C.round_to(w.logits, "bfloat16"), cu_rows=w.cu_rows,
                    draft_ids=w.draft_ids, temperature=w.temperature, top_k=w.top_k, top_p=w.top_p, min_p=w.min_p,
                    draft_kind=w.draft_kind, seed=w.seed, stream_id=w.stream_id, positions=w.positions, mask=None,
                    draft_logits=None, mode="ratio", logit_dtype="bfloat16")
        expected = oracle_outputs(case)
        for list_max in [256, 0]:
            got = run_abi(device_inputs(case), list_max=list_max)
            assert_same(got, expected, context=f"{case['name']} list_max={list_max}")


@pytest.mark.parametrize("vocab", range(1, 9))
def test_every_mask_of_a_uniform_row(vocab):
    """Every nonempty mask of a uniform row, with top-k 0, 1 or V and top-p
    1/4 ... 1, one request each (all tokens tie, so the kept set and the
    draw turn on ID order alone), against the oracle, with lists on and off."""
    combos = [(bits, k, p) for bits in range(1, 1 << vocab) for k in [0, 1, vocab] for p in [0.25, 0.5, 0.75, 1.0]]
    n = len(combos)
    case = C._case(f"masks_{vocab}", np.zeros((n, vocab)), np.arange(n + 1), np.empty((n, 0), np.int64),
                   top_k=[k for _, k, _ in combos], top_p=[p for _, _, p in combos],
                   seed=list(range(500, 500 + n)), mask=np.array([[bits] for bits, _, _ in combos], np.int32),
                   logit_dtype="float32")
    expected = oracle_outputs(case)
    for list_max in [256, 0]:
        assert_same(run_abi(device_inputs(case), list_max=list_max), expected, context=f"list_max={list_max}")


def test_temperature_only_batch_sizes_and_slot_permutation():
    case = C.workload_case("C2b")
    expected = oracle_outputs(case)
    whole = run_abi(device_inputs(case))
    assert_same(whole, expected)
    g = np.random.default_rng(5)
    order = g.permutation(case["cu_rows"].size - 1)
    perm = dict(case)
    for key in ["logits", "positions"]:
        perm[key] = case[key][order]
    for key in ["draft_ids", "temperature", "top_k", "top_p", "min_p", "draft_kind", "seed", "stream_id"]:
        perm[key] = case[key][order]
    got = run_abi(device_inputs(perm))
    np.testing.assert_array_equal(got[0], whole[0][order])
    for n in [1, 8]:
        sub = C.workload_case("C2b", list(range(n)))
        assert_same(run_abi(device_inputs(sub)), (x[:n] for x in expected), context=f"batch {n}")


def _oracle_case(rows, offsets, ids, params=None, rng=None, mask=None, draft_logits=None, mode="ratio",
                 dtype="float64"):
    rows = C.round_to(np.asarray(rows, dtype=np.float64), dtype)
    params = params or oracle.RequestParams()
    rng = rng or oracle.RngKey(1234, 3, np.arange(len(rows)))
    requests = len(offsets) - 1

    def per(v, kind=object):
        arr = np.asarray(v, dtype=object)
        return [arr.item()] * requests if arr.ndim == 0 else list(arr)

    case = C._case("adhoc", rows, offsets, C._drafts(ids, requests),
                   temperature=per(params.temperature), top_k=per(params.top_k), top_p=per(params.top_p),
                   min_p=per(params.min_p), draft_kind=per(params.draft_kind), seed=per(rng.seed),
                   stream=per(rng.stream_id), positions=rng.positions, mask=mask,
                   draft_logits=None if draft_logits is None else C.round_to(draft_logits, dtype), mode=mode,
                   logit_dtype=dtype)
    return case


def _run_fused(case, list_max=256, top_k_top_p=True):
    out, work = run_api(case, dispatch="fused", list_max=list_max, top_k_top_p=top_k_top_p)
    got = (out.tokens.cpu().numpy(), out.accepted_len.cpu().numpy(), out.status.cpu().numpy())
    assert_same(got, oracle_outputs(case))
    assert (out.path_used.cpu().numpy() == 1).all()
    return out, work.fallbacks()


def test_near_tie_scores_are_settled_in_fp64():
    seed, stream, position = 99, 5, 1000
    g0, g1 = oracle.gumbel(seed, stream, position, 0, 0), oracle.gumbel(seed, stream, position, 0, 1)
    rng = oracle.RngKey(seed, stream, [position])
    for eps in [1e-10, -1e-10]:
        case = _oracle_case(np.array([[0., g0 - g1 + eps]]), [0, 1], np.empty((1, 0)), rng=rng)
        out, fallbacks = _run_fused(case, list_max=0)
        assert out.tokens[0, 0].item() == (1 if eps > 0 else 0)
        assert fallbacks > 0
    case = _oracle_case(np.array([[0., g0 - g1]], np.float32), [0, 1], np.empty((1, 0)), rng=rng, dtype="float32")
    _, fallbacks = _run_fused(case, list_max=0)
    assert fallbacks > 0


def test_near_threshold_acceptance_is_exact():
    seed, stream, position = 4321, 2, 50
    u = oracle.uniform(seed, stream, position, 1, 0)
    rng = oracle.RngKey(seed, stream, [position, position + 1])
    for scale, accepted in [(1 + 1e-12, 1), (1 - 1e-12, 0)]:
        p = u * scale
        case = _oracle_case(np.array([[0., np.log(1 / p - 1)], [0., 0.]]), [0, 2], [[0]], rng=rng)
        for list_max in [256, 0]:
            out, _ = _run_fused(case, list_max=list_max)
            assert out.accepted_len[0].item() == accepted


def test_min_p_threshold_is_exact():
    rows = np.array([[0., -1.25, -3.]])
    for scale in [1 - 1e-9, 1 + 1e-9]:
        params = oracle.RequestParams(min_p=float(np.exp(-1.25)) * scale)
        for list_max in [256, 0]:
            for seed in range(20):
                _run_fused(_oracle_case(rows, [0, 1], np.empty((1, 0)), params=params,
                                        rng=oracle.RngKey(seed, 0, [seed])), list_max=list_max)


def test_top_k_selection_with_ties_and_large_k():
    g = np.random.default_rng(5)
    flat = np.zeros((1, 5000))
    for k in [1, 100, 2047, 2049, 4999]:
        for list_max in [256, 0]:
            _run_fused(_oracle_case(flat, [0, 1], np.empty((1, 0)), params=oracle.RequestParams(top_k=k),
                                    dtype="float32"), list_max=list_max)
    steps = np.round(g.normal(size=(3, 3000)) * 8) / 8
    for k in [257, 1000, 2999]:
        _run_fused(_oracle_case(steps, [0, 1, 3], [[-1], [7]], params=oracle.RequestParams(top_k=k, min_p=.001),
                                dtype="bfloat16"))


def test_top_p_over_the_full_row():
    g = np.random.default_rng(17)
    rows = g.normal(scale=3., size=(2, 151936))
    for k, p in [(0, .9), (1000, .8)]:
        _run_fused(_oracle_case(rows, [0, 2], [[5]], params=oracle.RequestParams(top_k=k, top_p=p, temperature=.7),
                                dtype="bfloat16"))
    flat = g.normal(scale=.5, size=(2, 20000))
    _run_fused(_oracle_case(flat, [0, 1, 2], np.empty((2, 0)), params=oracle.RequestParams(top_p=[.9, .3]),
                            dtype="float32"), list_max=0)


def test_top_p_boundary_on_exact_sums():
    g = np.random.default_rng(23)
    rows = g.normal(size=(1, 4096)) - 60
    rows[0, g.choice(4096, 50, replace=False)] = 0
    for count in [3, 40]:
        for list_max in [256, 0]:
            _run_fused(_oracle_case(rows, [0, 1], np.empty((1, 0)), params=oracle.RequestParams(top_p=count / 50),
                                    dtype="float32"), list_max=list_max)


def test_real_vocabulary_with_mask():
    g = np.random.default_rng(11)
    rows = g.normal(scale=3., size=(3, 151936))
    mask = workloads.packed_mask(g.random((3, 151936)) < .9)
    for k in [300, 5000]:
        _run_fused(_oracle_case(rows, [0, 3], [[17, 4]], params=oracle.RequestParams(top_k=k, temperature=.7),
                                mask=mask, dtype="bfloat16"))
    _run_fused(_oracle_case(rows[:1], [0, 1], np.empty((1, 0)), params=oracle.RequestParams(temperature=1.3),
                            dtype="bfloat16"))


def test_top_k_top_p_hint_never_changes_a_result():
    g = np.random.default_rng(7)
    offsets = np.array([0, 1, 3, 4, 6, 7, 8])
    rows = g.normal(scale=4., size=(offsets[-1], 2500))
    rows[7] = -np.inf
    params = oracle.RequestParams(temperature=[1., 0., .7, .6, 1., .8], top_k=[0, 0, 20, 0, 3, 0],
                                  top_p=[1., 1., .95, .9, 1., 1.], min_p=[0., 0., 0., .05, 0., 0.],
                                  draft_kind=["one_hot", "full", "one_hot", "one_hot", "one_hot", "one_hot"])
    ids = g.integers(0, 2500, size=(len(offsets) - 1, 1))
    q = g.normal(scale=2., size=rows.shape)
    for mode in ["ratio", "coupled"]:
        kw = dict(params=params, draft_logits=q) if mode == "ratio" else dict(
            params=dataclasses.replace(params, draft_kind=["one_hot"] * 6))
        case = _oracle_case(rows, offsets, ids, mode=mode, dtype="bfloat16", **kw)
        for hint in [True, False]:
            _run_fused(case, top_k_top_p=hint)


def test_batch_invariance_and_slice_count():
    g = np.random.default_rng(3)
    vocab, counts = 1000, [0, 3, 1, 2, 0]
    params = dict(temperature=[.7, 1., 0., .5, 1.2], top_k=[0, 20, 0, 400, 5], top_p=[.95, .9, 1., 1., .8],
                  min_p=[0., 0., 0., .05, 0.])
    rows = [g.normal(scale=3., size=(c + 1, vocab)) for c in counts]
    drafts = [g.integers(0, vocab, size=c) for c in counts]
    seeds, streams = [11, 22, 33, 44, 55], [1, 2, 3, 4, 5]
    positions = [np.arange(c + 1) + 40 * i for i, c in enumerate(counts)]

    def batch(order):
        sizes = [counts[i] + 1 for i in order]
        ids = np.full((len(order), 3), -1)
        for slot, i in enumerate(order):
            ids[slot, :counts[i]] = drafts[i]
        case = _oracle_case(np.concatenate([rows[i] for i in order]), np.concatenate([[0], np.cumsum(sizes)]), ids,
                            params=oracle.RequestParams(**{k: [v[i] for i in order] for k, v in params.items()}),
                            rng=oracle.RngKey([seeds[i] for i in order], [streams[i] for i in order],
                                              np.concatenate([positions[i] for i in order])), dtype="bfloat16")
        out, _ = run_api(case)
        return [(i, (out.tokens[slot].tolist(), out.accepted_len[slot].item(), out.status[slot].item()))
                for slot, i in enumerate(order)]

    together = dict(batch([0, 1, 2, 3, 4]))
    assert dict(batch([4, 2, 0, 3, 1])) == together
    for i in range(5):
        assert dict(batch([i]))[i] == together[i]
    for i, output in batch([0, 1, 2, 3, 4] * 9):  # more rows: a different cluster size
        assert output == together[i]


@pytest.mark.parametrize("ranks", [1, 2, 3, 5, 8, 16])
def test_results_do_not_depend_on_the_cluster_split(ranks, monkeypatch):
    monkeypatch.setenv("EXACTSAMPLE_CLUSTER", str(ranks))
    for entry in _large()[:4]:
        name, subset, digest, expected = entry
        case = golden_io.large_case(name, subset, digest)
        for list_max in [256, 0]:
            assert_same(run_abi(device_inputs(case), mode=case["mode"], list_max=list_max), expected,
                        context=f"{name} ranks={ranks}")
    for case, expected in SMALL[::7]:
        assert_same(run_abi(device_inputs(case), mode=case["mode"], list_max=0), expected, context=case["name"])


@pytest.mark.parametrize("stream", ["0", "1"])
def test_results_do_not_depend_on_the_row_mode(stream, monkeypatch):
    """Resident rows (slices kept in shared memory) and streamed rows (TMA ring,
    later passes from L2) give identical results."""
    monkeypatch.setenv("EXACTSAMPLE_STREAM", stream)
    for entry in _large():
        name, subset, digest, expected = entry
        case = golden_io.large_case(name, subset, digest)
        for list_max in [256, 0]:
            assert_same(run_abi(device_inputs(case), mode=case["mode"], list_max=list_max), expected,
                        context=f"{name} stream={stream}")
    for case, expected in SMALL[::3]:
        for list_max in [256, 0]:
            assert_same(run_abi(device_inputs(case), mode=case["mode"], list_max=list_max), expected,
                        context=case["name"])


@pytest.mark.parametrize("ring", ["2", "3", "4"])
def test_results_do_not_depend_on_the_ring_depth(ring, monkeypatch):
    """Streamed rows give identical results with a 2-, 3- or 4-stage TMA ring."""
    monkeypatch.setenv("EXACTSAMPLE_STREAM", "1")
    monkeypatch.setenv("EXACTSAMPLE_RING", ring)
    for entry in _large():
        name, subset, digest, expected = entry
        case = golden_io.large_case(name, subset, digest)
        assert_same(run_abi(device_inputs(case), mode=case["mode"]), expected, context=f"{name} ring={ring}")


def test_large_batch_is_invariant_to_how_it_is_split():
    """The reference's large-batch invariance check (tests/invariance/large_gpu.py):
    1,770 bf16 rows of the full vocabulary (a mix of sampling settings, and
    verification requests of 1 to 4 drafts) give each request the same
    outputs whether the batch runs whole or in three uneven parts."""
    import torch
    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey, plan, verify
    g = np.random.default_rng(1770)
    counts = []
    while sum(counts) < 1770:
        counts.append(int(min(g.integers(1, 6), 1770 - sum(counts))))
    requests = len(counts)
    cu = np.concatenate([[0], np.cumsum(counts)])
    rows = int(cu[-1])
    logits = torch.randn((rows, 151936), dtype=torch.float32, device="cuda") * 2.0
    peaks = torch.randint(0, 151936, (rows, 64), device="cuda")
    logits.scatter_add_(1, peaks, torch.rand((rows, 64), device="cuda") * 8 + 8)
    logits = logits.to(torch.bfloat16)
    max_draft = max(counts) - 1
    draft_np = np.full((requests, max_draft), -1, dtype=np.int64)
    for r, c in enumerate(counts):
        draft_np[r, :c - 1] = g.integers(0, 151936, c - 1)
    drafts = torch.as_tensor(draft_np, device="cuda")
    settings = [(0.6, 20, 0.95, 0.0), (1.0, 0, 1.0, 0.0), (0.8, 0, 0.9, 0.05), (0.0, 0, 1.0, 0.0), (1.2, 50, 1.0, 0.0)]
    pick = g.integers(0, len(settings), requests)
    f64 = lambda v: torch.as_tensor(np.asarray(v, np.float64), device="cuda")
    i64 = lambda v: torch.as_tensor(np.asarray(v, np.int64), device="cuda")
    params = CudaRequestParams(f64([settings[k][0] for k in pick]), i64([settings[k][1] for k in pick]),
                               f64([settings[k][2] for k in pick]), f64([settings[k][3] for k in pick]),
                               i64(np.zeros(requests)))
    seeds = i64(g.integers(-2**62, 2**62, requests))
    streams = i64(np.arange(requests))
    positions = i64(np.concatenate([np.arange(c) + int(g.integers(0, 30000)) for c in counts]))

    def run(r0, r1):
        a, b = int(cu[r0]), int(cu[r1])
        work = plan(b - a, r1 - r0, max_draft, 151936)
        out = work.allocate_output()
        sub = CudaRequestParams(*(x[r0:r1] for x in (params.temperature, params.top_k, params.top_p, params.min_p,
                                                     params.draft_kind)))
        verify(logits[a:b], i64(cu[r0:r1 + 1] - cu[r0]), drafts[r0:r1], params=sub,
               rng=CudaRngKey(seeds[r0:r1], streams[r0:r1], positions[a:b]), plan=work, out=out)
        work.synchronize()
        return out.tokens[:r1 - r0].cpu(), out.accepted_len[:r1 - r0].cpu(), out.status[:r1 - r0].cpu()

    whole = run(0, requests)
    assert (whole[2] == 0).all()
    cuts = [0, requests // 7, requests // 2 + 3, requests]
    parts = [run(a, b) for a, b in zip(cuts, cuts[1:])]
    for k in range(3):
        joined = torch.cat([part[k] for part in parts])
        assert torch.equal(joined, whole[k]), ["tokens", "accepted_len", "status"][k]
