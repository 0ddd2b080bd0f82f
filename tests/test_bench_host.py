"""CPU: bench.py's reference arm prints the driver's JSON line, and the append
oracle's semantics hold on constructed batches."""
import json

import pytest
import torch

import bench
from oracle import append_ref


def test_reference_arm_json_line(monkeypatch, capsys):
    """`bench.py --impl reference` at N=1: one JSON line with the contract's keys
    (the CPU samples are shortened for the test)."""
    real_chain, real_cfg1 = bench.cpu_chain_run, bench.cpu_config1_sample
    # one layer per step: the budget scales a step down to a bounded sample
    monkeypatch.setattr(bench, "cpu_chain_run",
                        lambda steps, warmup, budget_s: real_chain(steps, warmup, 1e-9))
    monkeypatch.setattr(bench, "cpu_config1_sample", lambda budget_s=0.0: real_cfg1(0.0))
    monkeypatch.setattr("sys.argv", ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"])
    bench.main()
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e", "cpu_config1"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["warmup"] >= 3
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["steps_timed"] == d["steps"]
    assert "first 1 of 32 layers" in d["cpu_baseline"]["sample"]
    assert "workload" in d["config"] and "whole host CPU" in d["config"]["scope"]


@pytest.mark.parametrize("page_size", [1, 16, 5])
def test_append_oracle_places_tokens_at_the_sequence_tail(page_size):
    """Every appended token of request b lands at sequence position
    seq_len[b] - n_b + j, on page kv_indices[kv_indptr[b] + p // page_size],
    slot p % page_size; nothing else is written."""
    g = torch.Generator().manual_seed(page_size)
    lens = [1, page_size, page_size + 1, 3 * page_size, 7]
    appended = [1, 1, page_size + 1, 2, 7]
    kp, ki, kl = [0], [], []
    next_page = 0
    for n in lens:
        pages = (n + page_size - 1) // page_size
        ki += list(range(next_page, next_page + pages))
        next_page += pages
        kp.append(kp[-1] + pages)
        kl.append(n - (pages - 1) * page_size)
    ai = [0]
    for a in appended:
        ai.append(ai[-1] + a)
    t = lambda x: torch.tensor(x, dtype=torch.int32)  # noqa: E731
    ai, kp, ki, kl = t(ai), t(kp), t(ki), t(kl)
    nnz = int(ai[-1])
    seq = append_ref.get_seq_lens(kp, kl, page_size)
    assert seq.tolist() == lens
    bi, pos = append_ref.get_batch_indices_positions(ai, seq, nnz)
    heads, hd = 2, 4
    key = torch.randn(nnz, heads * hd, generator=g)
    val = torch.randn(nnz, heads * hd, generator=g)
    cache = torch.zeros(next_page, 2, page_size, heads, hd)
    out = append_ref.append_paged_kv_cache(key, val, bi, pos, cache.clone(), ki, kp, kl)
    written = torch.zeros(next_page, page_size, dtype=torch.bool)
    for i in range(nnz):
        b = int(bi[i])
        j = i - int(ai[b])
        p = lens[b] - appended[b] + j
        assert int(pos[i]) == p
        page = int(ki[int(kp[b]) + p // page_size])
        assert torch.equal(out[page, 0, p % page_size], key[i].view(heads, hd))
        assert torch.equal(out[page, 1, p % page_size], val[i].view(heads, hd))
        written[page, p % page_size] = True
    assert int(out.abs().sum(dim=(1, 3, 4)).ne(0)[~written].sum()) == 0
