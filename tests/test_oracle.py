"""CPU: the oracle restatement against the reference's own outputs (golden fixtures and, where the reference
library is built, live runs), plus known answers of the number-format conversions."""

import numpy as np
import pytest
import torch

from oracle.oracle import Reference, Restatement, shard_sizes
from tests.helpers import DT_CODE, golden_cases, raw_from_torch

R = Restatement()


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c[0])
def test_restatement_matches_golden(case):
    name, meta, ins, outs = case
    code = DT_CODE[meta["dtype"]]
    op = meta["op"]
    if op == "all_reduce":
        got = R.fold_sum(ins, code, storage_round=True)
        for o in outs:
            assert np.array_equal(got, o)
    elif op == "reduce_scatter":
        got = R.reduce_scatter(ins, code, storage_round=True)
        for g, o in zip(got, outs):
            assert np.array_equal(g, o)
    elif op == "all_gather":
        got = R.all_gather(ins, meta["dim"])
        for o in outs:
            assert np.array_equal(got, o)
    elif op == "all_to_all":
        got = R.all_to_all(ins, meta["src_dim"], meta["dst_dim"])
        for g, o in zip(got, outs):
            assert g.shape == o.shape
            assert np.array_equal(g, o)
    else:
        raise AssertionError(op)


def test_shard_sizes_rule():
    # Placement::GetShardSizeForAllRank: first L % n ranks get one more
    assert shard_sizes(9, 2) == [5, 4]
    assert shard_sizes(8, 2) == [4, 4]
    assert shard_sizes(11, 4) == [3, 3, 3, 2]
    assert shard_sizes(64, 8) == [8] * 8


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_format_conversion_matches_torch(dtype):
    g = torch.Generator().manual_seed(7)
    x = torch.cat([torch.randn(20000, generator=g) * s for s in (1e-8, 1e-5, 1e-2, 1.0, 1e3, 6e4, 1e38)])
    x = torch.cat([x, torch.tensor([0.0, -0.0, 65504.0, 65520.0, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                                    float("inf"), -float("inf")])])
    want = raw_from_torch(x.to(dtype))
    f = R.lib.oracle_f32_to_bf16 if dtype == torch.bfloat16 else R.lib.oracle_f32_to_f16
    got = np.array([f(float(v)) for v in x.tolist()], dtype=np.uint16)
    assert np.array_equal(got, want)
    back = R.lib.oracle_bf16_to_f32 if dtype == torch.bfloat16 else R.lib.oracle_f16_to_f32
    vals = np.array([back(int(b)) for b in want[:5000]], dtype=np.float32)
    assert np.array_equal(vals, x[:5000].to(dtype).float().numpy())


def test_fp32_accumulate_mode_differs_only_by_rounding():
    # storage_round=False is the CUDA kernels' default: fp32 accumulation, one rounding at the end
    g = torch.Generator().manual_seed(3)
    ins = [raw_from_torch(torch.randn(5000, generator=g).to(torch.bfloat16)) for _ in range(8)]
    a = R.fold_sum(ins, 1, storage_round=True)
    b = R.fold_sum(ins, 1, storage_round=False)
    fa = (a.astype(np.uint32) << 16).view(np.float32)
    fb = (b.astype(np.uint32) << 16).view(np.float32)
    assert np.allclose(fa, fb, rtol=2e-2, atol=2e-2 * np.sqrt(np.mean(fa * fa)))


@pytest.mark.skipif(not Reference.available(), reason="reference library not built here")
@pytest.mark.parametrize("n", [2, 4, 8])
def test_restatement_matches_live_reference(n):
    ref = Reference()
    g = torch.Generator().manual_seed(n)
    for dt, code in [(torch.float32, 0), (torch.bfloat16, 1), (torch.float16, 2)]:
        ins = [raw_from_torch(torch.randn(3 * n + 5, 7, generator=g).to(dt)) for _ in range(n)]
        outs, _ = ref.all_reduce(ins, code)
        assert np.array_equal(R.fold_sum(ins, code, True).reshape(-1), outs[0])
        lens = shard_sizes(3 * n + 5, n)
        parts = [raw_from_torch(torch.randn(l, 2 * n + 3, generator=g).to(dt)) for l in lens]
        outs, _ = ref.all_to_all(parts, code, 0, 1)
        for a, b in zip(R.all_to_all(parts, 0, 1), outs):
            assert np.array_equal(a, b)


@pytest.mark.skipif(not Reference.available(), reason="reference library not built here")
def test_restatement_matches_live_reference_on_random_cases():
    """Random group sizes, shapes, dims and dtypes, restricted to what the reference accepts (its debug asserts
    end the process otherwise): every collective of the restatement equals the reference's own output."""
    hyp = pytest.importorskip("hypothesis")
    st = pytest.importorskip("hypothesis.strategies")
    ref = Reference()

    @hyp.settings(max_examples=60, deadline=None)
    @hyp.given(st.data())
    def check(data):
        n = data.draw(st.integers(2, 8))
        code = data.draw(st.sampled_from([0, 1, 2]))
        dt = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}[code]
        op = data.draw(st.sampled_from(["all_reduce", "reduce_scatter", "all_gather", "all_to_all"]))
        ndim = data.draw(st.integers(1 if op != "all_to_all" else 2, 4))
        shape = [data.draw(st.integers(1, 6)) for _ in range(ndim)]
        g = torch.Generator().manual_seed(data.draw(st.integers(0, 2 ** 31 - 1)))
        if op in ("all_reduce", "reduce_scatter"):
            count = int(np.prod(shape)) * (n if op == "reduce_scatter" else 1)
            ins = [raw_from_torch(torch.randn(count, generator=g).to(dt)) for _ in range(n)]
            if op == "all_reduce":
                outs, _ = ref.all_reduce(ins, code)
                want = [R.fold_sum(ins, code, True).reshape(-1)] * n
            else:
                outs, _ = ref.reduce_scatter(ins, code)
                want = R.reduce_scatter(ins, code, True)
            for a, b in zip(want, outs):
                assert np.array_equal(np.asarray(a).reshape(-1), b.reshape(-1))
            return
        dim = data.draw(st.integers(0, ndim - 1))
        length = data.draw(st.integers(n, 3 * n + 2))
        lens = shard_sizes(length, n)
        if op == "all_gather":
            parts = []
            for l in lens:
                s = list(shape)
                s[dim] = l
                parts.append(raw_from_torch(torch.randn(*s, generator=g).to(dt)))
            outs, _ = ref.all_gather(parts, code, dim)
            want = R.all_gather(parts, dim)
            for b in outs:
                assert np.array_equal(want, b)
            return
        dst = data.draw(st.sampled_from([d for d in range(ndim) if d != dim]))
        parts = []
        for l in lens:
            s = list(shape)
            s[dim] = l
            s[dst] = max(s[dst], n) + data.draw(st.integers(0, 3)) if l == lens[0] else s[dst]
            parts.append(s)
        dst_len = parts[0][dst]
        tensors = []
        for s in parts:
            s = list(s)
            s[dst] = dst_len
            tensors.append(raw_from_torch(torch.randn(*s, generator=g).to(dt)))
        outs, _ = ref.all_to_all(tensors, code, dim, dst)
        for a, b in zip(R.all_to_all(tensors, dim, dst), outs):
            assert np.array_equal(a, b)

    check()
