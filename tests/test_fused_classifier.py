"""GPU parity of the fused variant: the tcgen05 classifier GEMM (logits =
hidden . wcls^T, bf16 in, fp32 accumulate) and the sampling of its rows.

Bars:
  * logits against a plain PyTorch fp32 matmul of the same bf16 operands
    (exact products, only the summation order differs): |diff| <= LOGIT_ATOL
    plus LOGIT_RTOL times the sum of |products| of the entry;
  * ids, states and flags: identical to sampler_batched() run on the fused
    call's own logits (the epilogue statistics only replace the sampler's
    first pass), and those ids pass the end-to-end rule against the oracle;
  * the final RMSNorm prologue: within one bf16 rounding of a PyTorch fp32
    rmsnorm (the sum of squares is a tree sum here, serial in the reference).
"""
import numpy as np
import pytest
import torch

from test_gpu_parity import check_e2e

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
LOGIT_ATOL = 1e-5
LOGIT_RTOL = 2e-6


def operands(B, D, V, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(B, D, generator=g).to(torch.bfloat16)
    w = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16)
    return h.to(DEV), w.to(DEV)


def fused(pkg, h, w, temp, topp, seeds, topp_rows=None, temp_rows=None):
    B, V = h.shape[0], w.shape[0]
    st = torch.from_numpy(np.asarray(seeds, np.uint64).view(np.int64).copy()).to(DEV)
    logits = torch.empty(B, V, device=DEV)
    flags = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    tr = None if topp_rows is None else torch.from_numpy(np.asarray(topp_rows, np.float32)).to(DEV)
    te = None if temp_rows is None else torch.from_numpy(np.asarray(temp_rows, np.float32)).to(DEV)
    ids = pkg.classifier_sample_fused(h, w, temp, topp, st, topp_rows=tr, temperature_rows=te, logits_out=logits,
                                      row_flags=flags)
    torch.cuda.synchronize()
    return dict(ids=ids.cpu().numpy(), states=st.cpu().numpy().view(np.uint64), logits=logits,
                flags=flags.cpu().numpy())


def unfused(pkg, logits, temp, topp, seeds, topp_rows=None, temp_rows=None):
    B = logits.shape[0]
    st = torch.from_numpy(np.asarray(seeds, np.uint64).view(np.int64).copy()).to(DEV)
    flags = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    tr = None if topp_rows is None else torch.from_numpy(np.asarray(topp_rows, np.float32)).to(DEV)
    te = None if temp_rows is None else torch.from_numpy(np.asarray(temp_rows, np.float32)).to(DEV)
    ids = pkg.sample_batched(logits, temp, topp, st, topp_rows=tr, temperature_rows=te, row_flags=flags)
    torch.cuda.synchronize()
    return dict(ids=ids.cpu().numpy(), states=st.cpu().numpy().view(np.uint64), flags=flags.cpu().numpy())


def check_logits(h, w, logits):
    ref = h.float() @ w.float().t()
    bound = h.float().abs() @ w.float().abs().t()
    err = (logits - ref).abs()
    ok = err <= LOGIT_ATOL + LOGIT_RTOL * bound
    assert bool(ok.all()), f"max |diff| {err.max().item():.3g}, worst ratio {(err / (bound + 1e-30)).max().item():.3g}"


# (B, D, V): the decode shape with fewer rows, then tails in every dimension
# (rows % 128, dim % 64, vocab % 256); one or two rows take the CUDA-core
# GEMV (dim % 256 tails included), three rows the smallest tensor-core tile
SHAPES = [(256, 4096, 32000), (300, 4096, 4064), (130, 520, 32000), (1, 64, 256), (1, 4096, 32000),
          (2, 4104, 32000), (2, 520, 4064), (3, 4096, 32000)]


@pytest.mark.parametrize("B,D,V", SHAPES)
def test_fused_logits_and_ids(pkg, orc, B, D, V):
    h, w = operands(B, D, V, seed=4 + B)
    seeds = pkg.workloads.row_seeds(B)
    topps = np.where(np.arange(B) % 2 == 0, 0.9, 0.95).astype(np.float32)
    out = fused(pkg, h, w, 0.8, 0.9, seeds, topp_rows=topps)
    check_logits(h, w, out["logits"])
    ref = unfused(pkg, out["logits"], 0.8, 0.9, seeds, topp_rows=topps)
    assert np.array_equal(out["ids"], ref["ids"])
    assert np.array_equal(out["states"], ref["states"])
    assert np.array_equal(out["flags"], ref["flags"])
    n = min(B, 64)
    x = out["logits"][:n].cpu().numpy()
    ref_ids, ref_st, ref_p = orc.sample_batch(x, 0.8, 0.9, seeds[:n], topp_rows=topps[:n], probs_out=True)
    assert np.array_equal(out["states"][:n], ref_st)
    check_e2e(orc, out["ids"][:n], ref_ids, ref_p, seeds[:n], topps[:n])


@pytest.mark.parametrize("B", [200, 2])
def test_fused_greedy_and_mixed_rows(pkg, orc, B):
    D, V = 1024, 32000
    h, w = operands(B, D, V, seed=99)
    temps = np.where(np.arange(B) % 4 == 0, 0.0, 0.7).astype(np.float32)
    topps = np.where(np.arange(B) % 3 == 0, 1.0, 0.9).astype(np.float32)
    seeds = pkg.workloads.row_seeds(B, seed=7)
    out = fused(pkg, h, w, 0.7, 0.9, seeds, topp_rows=topps, temp_rows=temps)
    check_logits(h, w, out["logits"])
    ref = unfused(pkg, out["logits"], 0.7, 0.9, seeds, topp_rows=topps, temp_rows=temps)
    assert np.array_equal(out["ids"], ref["ids"]) and np.array_equal(out["states"], ref["states"])
    x = out["logits"].cpu().numpy()
    greedy = np.nonzero(temps == 0.0)[0]
    assert [int(out["ids"][r]) for r in greedy] == [orc.argmax(x[r]) for r in greedy]


def test_fused_all_greedy(pkg, orc):
    B, D, V = 64, 4096, 32000
    h, w = operands(B, D, V, seed=5)
    out = fused(pkg, h, w, 0.0, 0.9, pkg.workloads.row_seeds(B))
    x = out["logits"].cpu().numpy()
    assert out["ids"].tolist() == [orc.argmax(r) for r in x]


def test_fused_rejects_bad_shapes(pkg):
    h, w = operands(4, 64, 100, seed=1)  # vocab not a multiple of 32
    with pytest.raises(pkg.SamplerError):
        pkg.classifier_sample_fused(h, w, 1.0, 0.9, torch.zeros(4, dtype=torch.int64, device=DEV))


def test_rmsnorm_prologue_and_decode_step(pkg):
    """Final RMSNorm (llama2.c rmsnorm) into bf16, then the fused classifier:
    the normalized rows are within one bf16 rounding of a PyTorch fp32
    reference, and the decode step's ids equal classifier_sample_fused on
    those rows."""
    B, D, V = 96, 4096, 32000
    g = torch.Generator().manual_seed(31)
    x = (torch.randn(B, D, generator=g) * 3.0).to(DEV)
    nw = (1.0 + 0.1 * torch.randn(D, generator=g)).to(DEV)
    w = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    h = pkg.rmsnorm_bf16(x, nw)
    torch.cuda.synchronize()
    ref = nw * (x * (1.0 / torch.sqrt((x * x).mean(dim=1, keepdim=True) + 1e-5)))
    ref_b = ref.to(torch.bfloat16).float()
    diff = (h.float() - ref_b).abs()
    ulp = ref_b.abs() * 2.0 ** -7  # one bf16 ulp (8-bit significand)
    assert bool((diff <= ulp + 1e-30).all()), f"max diff {diff.max().item():.3g}"
    assert float((diff == 0).float().mean()) > 0.999  # nearly all bit-identical
    seeds = pkg.workloads.row_seeds(B)
    st1 = torch.from_numpy(seeds.view(np.int64).copy()).to(DEV)
    st2 = st1.clone()
    ids1 = pkg.classifier_rmsnorm_sample_fused(x, nw, w, 0.8, 0.9, st1)
    ids2 = pkg.classifier_sample_fused(h, w, 0.8, 0.9, st2)
    torch.cuda.synchronize()
    assert torch.equal(ids1, ids2) and torch.equal(st1, st2)


def test_device_resident_decode_loop_in_a_cuda_graph(pkg):
    """A decode loop whose next input is gathered on the device from the
    sampled ids (no host sync per token), eagerly and captured once in a CUDA
    graph and replayed: same ids and states at every step."""
    B, D, V, steps = 48, 256, 2048, 5
    g = torch.Generator().manual_seed(41)
    table = (torch.randn(V, D, generator=g) * 2.0).to(DEV)
    nw = (1.0 + 0.1 * torch.randn(D, generator=g)).to(DEV)
    wcls = table.to(torch.bfloat16)  # shared classifier / embedding weights
    seeds = torch.from_numpy(pkg.workloads.row_seeds(B).view(np.int64).copy()).to(DEV)
    ids0 = torch.arange(B, dtype=torch.int32, device=DEV) * 37 % V

    def run(step_fn, x, st, ids):
        out = []
        for _ in range(steps):
            step_fn(x, st, ids)
            out.append(ids.clone())
        torch.cuda.synchronize()
        return torch.stack(out).cpu(), st.cpu()

    def step(x, st, ids):
        pkg.classifier_rmsnorm_sample_fused(x, nw, wcls, 0.9, 0.9, st, out_ids=ids)
        pkg.gather_rows(table, ids, out=x)

    x = pkg.gather_rows(table, ids0)
    st = seeds.clone()
    ids = torch.empty(B, dtype=torch.int32, device=DEV)
    want_ids, want_st = run(step, x, st, ids)

    x = pkg.gather_rows(table, ids0)
    st = seeds.clone()
    ids = torch.empty(B, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(x, st, ids)
    x.copy_(pkg.gather_rows(table, ids0))
    st.copy_(seeds)
    torch.cuda.synchronize()
    got_ids, got_st = run(lambda *_: graph.replay(), x, st, ids)
    assert torch.equal(got_ids, want_ids) and torch.equal(got_st, want_st)
    assert len(set(want_ids[-1].tolist())) > 1  # the loop really samples


def test_fused_full_decode_batch_seeded_operands(pkg, orc):
    """The fused workload as configured: 8192 hidden states of dim 4096
    (seed-4 numpy operands, bf16) against wcls [32000, 4096], T = 0.8,
    topp 0.9.  Logits against an fp32 matmul of the same bf16 operands in row
    blocks; ids, states and flags equal sampler_batched on the fused call's own
    logits for every row; 1024 rows spread over the batch pass the end-to-end
    rule against the oracle."""
    f = pkg.workloads.fused()
    h = torch.from_numpy(f["hidden"].view(np.int16)).view(torch.bfloat16).to(DEV)
    w = torch.from_numpy(f["wcls"].view(np.int16)).view(torch.bfloat16).to(DEV)
    B, V = h.shape[0], w.shape[0]
    assert (B, h.shape[1], V) == (8192, 4096, 32000)
    seeds = pkg.workloads.row_seeds(B, seed=f["seed"])
    out = fused(pkg, h, w, f["temperature"], f["topp"], seeds)
    for b0 in range(0, B, 1024):
        check_logits(h[b0:b0 + 1024], w, out["logits"][b0:b0 + 1024])
    ref = unfused(pkg, out["logits"], f["temperature"], f["topp"], seeds)
    assert np.array_equal(out["ids"], ref["ids"])
    assert np.array_equal(out["states"], ref["states"])
    assert np.array_equal(out["flags"], ref["flags"])
    rows = np.arange(0, B, 8)
    x = out["logits"][torch.from_numpy(rows).to(DEV)].cpu().numpy()
    ref_ids, ref_st, ref_p = orc.sample_batch(x, f["temperature"], f["topp"], seeds[rows], probs_out=True)
    assert np.array_equal(out["states"][rows], ref_st)
    check_e2e(orc, out["ids"][rows], ref_ids, ref_p, seeds[rows], np.full(len(rows), f["topp"]))


def test_device_logits_through_dump_files(pkg, orc, tmp_path):
    """The classifier's device logits written as the reference's -DDUMP_LOGITS
    files (a raw fp32 row per step, the JSON id list) and read back the way its
    analysis script reads them: the same bits, and the ids the fused call
    sampled from them."""
    B, D, V = 6, 4096, 32000
    h, w = operands(B, D, V, seed=77)
    logits = pkg.classifier_logits(h, w)
    seeds = pkg.workloads.row_seeds(B)
    st = torch.from_numpy(seeds.view(np.int64).copy()).to(DEV)
    ids = pkg.classifier_sample_fused(h, w, 0.8, 0.9, st)
    torch.cuda.synchronize()
    d = pkg.dumps
    lp, ip = tmp_path / "ours.bin", tmp_path / "ids.json"
    for step in range(B):  # one decode step per row, as the generate loop dumps them
        d.append_logits(lp, logits[step], first=(step == 0))
        d.append_token_ids(ip, ids[step:step + 1], first=(step == 0))
    back = np.fromfile(lp, dtype=np.float32).reshape(-1, V)
    assert np.array_equal(back.view(np.uint32), logits.cpu().numpy().view(np.uint32))
    assert np.array_equal(d.load_logits(lp, V), back)
    import json
    assert json.load(open(ip)) == ids.cpu().numpy().tolist()
    ref_ids, _, ref_p = orc.sample_batch(back, 0.8, 0.9, seeds, probs_out=True)
    check_e2e(orc, ids.cpu().numpy(), ref_ids, ref_p, seeds, np.full(B, 0.9))


@pytest.mark.parametrize("B,D", [(1, 4096), (2, 4096), (1, 520), (2, 4104)])
def test_rmsnorm_folded_into_decode_classifier(pkg, B, D):
    """At decode batches (one or two rows) the final RMSNorm is folded into
    the classifier kernel: the call launches one kernel fewer than
    rmsnorm_bf16 followed by classifier_sample_fused, and gives the same
    logits bit for bit (the fold repeats the norm kernel's arithmetic in its
    order), hence the same ids and states."""
    V = 32000
    g = torch.Generator().manual_seed(61 + B + D)
    x = (torch.randn(B, D, generator=g) * 3.0).to(DEV)
    nw = (1.0 + 0.1 * torch.randn(D, generator=g)).to(DEV)
    w = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    seeds = pkg.workloads.row_seeds(B)
    st1 = torch.from_numpy(seeds.view(np.int64).copy()).to(DEV)
    st2 = st1.clone()
    lg1 = torch.empty(B, V, device=DEV)
    lg2 = torch.empty(B, V, device=DEV)
    ids1 = pkg.classifier_rmsnorm_sample_fused(x, nw, w, 0.8, 0.9, st1, logits_out=lg1)
    n_fold = pkg.last_launch_count()
    h = pkg.rmsnorm_bf16(x, nw)
    n_norm = pkg.last_launch_count()
    ids2 = pkg.classifier_sample_fused(h, w, 0.8, 0.9, st2, logits_out=lg2)
    n_fused = pkg.last_launch_count()
    torch.cuda.synchronize()
    assert n_fold == n_norm + n_fused - 1
    assert torch.equal(lg1.view(torch.int32), lg2.view(torch.int32))
    assert torch.equal(ids1, ids2) and torch.equal(st1, st2)
    # the logits against an fp32 matmul of the fp32-normalized rows: within the
    # bf16 rounding of the operand (2^-8 relative per product, summed)
    ref_h = nw * (x * (1.0 / torch.sqrt((x * x).mean(dim=1, keepdim=True) + 1e-5)))
    ref = ref_h @ w.float().t()
    bound = ref_h.abs() @ w.float().abs().t()
    assert bool(((lg1 - ref).abs() <= 2.0 ** -8 * bound + 1e-5).all())
