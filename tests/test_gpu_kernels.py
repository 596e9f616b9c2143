"""GPU parity of each kernel of the C ABI against the CPU oracle.

Integer work (routing ids, capacity drops, packed layouts) must match bit
for bit.  Floating point tolerances:
  * router ids and weights: bit-exact against the oracle's selection over
    torch's CUDA softmax (the reference's GPU routing); <= 1 bf16 ulp
    against the oracle's own numpy softmax;
  * expert rows / layer outputs: max |diff| <= 2^-7 * max|ref| and
    mean |diff| <= 2e-4 * max|ref| against the oracle (fp32 accumulation
    order differs; the rounding points are the same).  The reference's own
    Triton path, whose outputs these kernels equal bit for bit
    (test_gpu_reference_triton.py), sits at up to 0.0056 * max|ref| from the
    oracle on the 235B shape;
  * combine: bit-exact (same fp32 slot-order sum).
"""

import functools

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200 as pkg
import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, ops
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def assert_close_rel(got: np.ndarray, ref: np.ndarray, max_rel=2.0 ** -7, mean_rel=2e-4):
    scale = float(np.abs(ref).max()) or 1.0
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    assert diff.max() <= max_rel * scale, (diff.max(), scale)
    assert diff.mean() <= mean_rel * scale, (diff.mean(), scale)


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0, "a kernel reported a timeout or bad index"


def cuda_probs(logits: torch.Tensor) -> np.ndarray:
    """torch's CUDA softmax of the logits (the reference's moe.py:872 on a GPU)."""
    return torch.softmax(logits.to(DEV), dim=-1, dtype=torch.float32).cpu().numpy()


@pytest.mark.parametrize("tokens,experts,top_k", [(1, 128, 8), (7, 8, 2), (512, 128, 8),
                                                  (8192, 128, 8), (33, 4, 2), (64, 1024, 8),
                                                  (5, 40, 32)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_fp32_logits(tokens, experts, top_k, renorm):
    logits = wl.uniform_logits(tokens, experts, seed=tokens + experts)
    w, ids = ops.route_topk(logits.to(DEV), top_k, renorm)
    # Selection and renormalisation of the oracle over torch's CUDA softmax:
    # bit-exact ids and weights.
    ref_w, ref_ids = mo.route_from_probs(cuda_probs(logits), top_k, renorm)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_array_equal(bits(w), mo.bf16_bits(ref_w))
    # The oracle's own softmax (numpy exp): same ids, weights within 1 bf16 ulp.
    o_w, o_ids = mo.route_topk(logits.numpy(), top_k, renorm)
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)
    ulp = np.abs(bits(w).astype(np.int32) - mo.bf16_bits(o_w).astype(np.int32))
    assert ulp.max() <= 1


def test_router_bf16_logits_golden_outside_ties(golden):
    """The CPU-recorded reference golden: equal outside tie tokens (its CPU
    torch.topk orders ties differently from the CUDA one matched here)."""
    logits = torch.from_numpy(golden["route_bf16_logits"].astype(np.int16)).view(
        torch.bfloat16).reshape(256, 128)
    w, ids = ops.route_topk(logits.to(DEV), 8, True)
    ties = mo.tie_tokens(logits.float().numpy(), 8)
    np.testing.assert_array_equal(ids.cpu().numpy()[~ties], golden["route_bf16_ids"][~ties])


def test_router_reference_golden_fp32(golden):
    logits = torch.from_numpy(golden["route_f32_logits"])
    w, ids = ops.route_topk(logits.to(DEV), 8, True)
    np.testing.assert_array_equal(ids.cpu().numpy(), golden["route_f32_ids"])
    ulp = np.abs(bits(w).astype(np.int32) - golden["route_f32_w"].astype(np.int32))
    assert ulp.max() <= 1


def _check_pack(ids_np, num_experts, num_local, expert_start=0, local_index=None,
                capacity=None, expert_base=None):
    ids = torch.from_numpy(ids_np.copy()).to(DEV)
    w = torch.rand(ids.shape, device=DEV).to(torch.bfloat16)
    w_before = w.clone()
    li = None if local_index is None else torch.from_numpy(local_index).to(DEV)
    eb = None if expert_base is None else torch.from_numpy(expert_base).to(DEV)
    stats = torch.zeros(2, device=DEV, dtype=torch.int64)
    p = ops.pack_routes(ids.view(-1), w.view(-1), num_experts, num_local, local_index=li,
                        expert_start=expert_start, expert_base=eb, capacity=capacity,
                        stats=stats)
    torch.cuda.synchronize()
    ref_w, ref_ids, keep = mo.apply_capacity(w_before.float().cpu().numpy(), ids_np,
                                             num_experts, capacity, expert_base)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_array_equal(w.float().cpu().numpy(), ref_w)
    lay = mo.pack(ref_ids.reshape(-1), num_experts, num_local, expert_start, local_index)
    assert p.row_capacity == mo.row_capacity(ids_np.size, num_local)
    np.testing.assert_array_equal(p.row_route.cpu().numpy(), lay["row_route"])
    np.testing.assert_array_equal(p.route_row.cpu().numpy(), lay["route_row"])
    np.testing.assert_array_equal(p.combine_rows.cpu().numpy(), lay["combine_rows"])
    np.testing.assert_array_equal(p.tile_expert.cpu().numpy(), lay["tile_expert"])
    np.testing.assert_array_equal(p.expert_offsets.cpu().numpy(), lay["expert_offsets"])
    np.testing.assert_array_equal(p.expert_counts.cpu().numpy(), lay["expert_counts"])
    counters = p.counters.cpu().numpy()
    n_m = len(lay["mtiles"])
    assert counters[_lib.CNT_PADDED_ROWS] == lay["padded_rows"]
    assert counters[_lib.CNT_MTILES] == n_m
    assert counters[_lib.CNT_LOCAL_KEPT] == lay["local_kept"]
    assert counters[_lib.CNT_DROPPED] == int((~keep).sum())
    np.testing.assert_array_equal(p.mtiles.cpu().numpy()[:n_m], lay["mtiles"])
    n_c = len(lay["chunks"])
    assert counters[_lib.CNT_CHUNKS] == n_c
    np.testing.assert_array_equal(p.chunks.cpu().numpy()[:n_c], lay["chunks"])
    assert stats.tolist() == [lay["local_kept"], int((~keep).sum())]


@pytest.mark.parametrize("tokens,experts,top_k", [(1, 128, 8), (16, 128, 8), (512, 128, 8),
                                                  (8192, 128, 8), (3, 8, 2), (1000, 64, 6)])
def test_pack_full_placement(tokens, experts, top_k):
    logits = wl.uniform_logits(tokens, experts, seed=3 * tokens + 1)
    _, ids = mo.route_topk(logits.numpy(), top_k, True)
    _check_pack(ids, experts, experts)


@pytest.mark.parametrize("rank", [0, 3])
def test_pack_contiguous_shard_and_round_robin(rank):
    logits = wl.uniform_logits(512, 128, seed=7)
    _, ids = mo.route_topk(logits.numpy(), 8, True)
    _check_pack(ids, 128, 32, expert_start=32 * rank)
    local_index = np.array([(e // 4 if e % 4 == rank else -1) for e in range(128)])
    _check_pack(ids, 128, 32, local_index=local_index)


def test_pack_invalid_and_sentinel_ids():
    ids = np.array([[-1, 0], [1, 2], [3, 4], [4, 4]], dtype=np.int64)
    _check_pack(ids, 4, 2, local_index=np.array([0, -1, -1, 1]))
    _check_pack(ids, 4, 4)


@pytest.mark.parametrize("capacity", [1, 5, 640])
def test_pack_capacity(capacity):
    logits = wl.zipf_logits(8192, 128, seed=5)
    _, ids = mo.route_topk(logits.numpy(), 8, True)
    _check_pack(ids, 128, 128, capacity=capacity)


def test_pack_capacity_with_expert_base_and_shard():
    logits = wl.zipf_logits(2048, 128, seed=9)
    _, ids = mo.route_topk(logits.numpy(), 8, True)
    base = np.random.default_rng(0).integers(0, 200, size=128).astype(np.int32)
    _check_pack(ids, 128, 32, expert_start=64, capacity=160, expert_base=base)


def test_capacity_zipf_matches_reference_golden(golden):
    logits = wl.zipf_logits(8192, 128, seed=5, alpha=1.2)
    w, ids = ops.route_topk(logits.to(DEV), 8, True)
    p = ops.pack_routes(ids.view(-1), w.view(-1), 128, 128, capacity=640)
    np.testing.assert_array_equal(ids.cpu().numpy(), golden["cap_zipf_ids"].astype(np.int64))
    assert int(p.counters[_lib.CNT_DROPPED]) == int(golden["cap_zipf_dropped"][0])
    ulp = np.abs(bits(w).astype(np.int32) - golden["cap_zipf_w"].astype(np.int32))
    assert ulp.max() <= 1


def test_combine_known_answers():
    y = torch.tensor([[1.0] * 16, [0.00390625] * 16], dtype=torch.bfloat16, device=DEV)
    out = ops.combine(y, torch.tensor([0, 1], device=DEV), 1, 2, torch.float32)
    assert out.dtype == torch.float32
    assert torch.equal(out.cpu(), torch.full((1, 16), 1.00390625))
    vals = torch.tensor([0.043701171875, 0.037109375, -0.0047607421875, -0.00506591796875,
                         -4.423782229423523e-09, -0.001953125, 0.005859375,
                         -0.01068115234375], dtype=torch.bfloat16)
    y = vals.unsqueeze(1).expand(8, 16).contiguous().to(DEV)
    out = ops.combine(y, torch.arange(8, device=DEV), 1, 8, torch.float64, accum_f64=True)
    assert torch.equal(out.cpu(), vals.double().sum(dim=0, keepdim=True).expand(1, 16))
    torch.manual_seed(23)
    packed = torch.randn(9, 32, dtype=torch.bfloat16)
    rr = torch.tensor([3, 0, 9, 7, 2, 9, 8, 1, 4, 9, 6, 5], dtype=torch.int32)
    expect = torch.cat((packed, torch.zeros_like(packed[:1])))[rr.long()].reshape(
        3, 4, 32).float().sum(dim=1).bfloat16()
    got = ops.combine(packed.to(DEV), rr.to(DEV), 3, 4)
    assert torch.equal(got.cpu(), expect)


@functools.lru_cache(maxsize=2)
def _weights(shape, seed):
    return wl.expert_weights(shape, seed=seed)


def _expert_case(shape, tokens, engine, seed, logits_kind="uniform", capacity=None,
                 packed_rows=False):
    w13, w2 = _weights(shape, 11)
    x = wl.hidden_states(tokens, shape.hidden, seed=seed + 1)
    if logits_kind == "uniform":
        logits = wl.uniform_logits(tokens, shape.num_experts, seed=seed + 2)
    else:
        logits = wl.zipf_logits(tokens, shape.num_experts, seed=seed + 2)
    res = mo.moe_forward(x.float().numpy(), logits.numpy(), w13.float().numpy(),
                         w2.float().numpy(), shape.top_k, True, capacity=capacity,
                         probs=cuda_probs(logits))
    xd, w13d, w2d = x.to(DEV), w13.to(DEV), w2.to(DEV)
    w, ids = ops.route_topk(logits.to(DEV), shape.top_k, True)
    p = ops.pack_routes(ids.view(-1), w.view(-1), shape.num_experts, shape.num_experts,
                        capacity=capacity)
    if engine == _lib.ENGINE_STREAM:
        act = ops.expert_gate_up(engine, xd, None, w13d, p, shape.top_k)
    elif packed_rows or engine in (_lib.ENGINE_TCGEN05_PAIR, _lib.ENGINE_TCGEN05_TALL):
        xp = ops.gather_rows(xd, p, shape.top_k)
        act = ops.expert_gate_up(engine, xd, xp, w13d, p, shape.top_k)
    else:
        # One-SM tcgen05 engines gather token rows inside their TMA loads.
        act = ops.expert_gate_up(engine, xd, None, w13d, p, shape.top_k)
    y = ops.expert_down(engine, act, w2d, p, w.view(-1), tokens)
    out = ops.combine(y, p.combine_rows, tokens, shape.top_k)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), res["ids"])
    computed = p.combine_rows.cpu().numpy() < p.num_routes
    assert_close_rel(y.float().cpu().numpy()[computed], res["y"][computed])
    assert_close_rel(out.float().cpu().numpy(), res["output"])
    return out


SMALL = wl.LayerShape("small", 128, 256, 8, 2)
TINY = wl.LayerShape("tiny", 32, 64, 128, 8)
A = wl.QWEN3_30B_A3B


ENGINES = [_lib.ENGINE_STREAM, _lib.ENGINE_TCGEN05, _lib.ENGINE_TCGEN05_WIDE,
           _lib.ENGINE_TCGEN05_SWAP, _lib.ENGINE_TCGEN05_PAIR, _lib.ENGINE_TCGEN05_TALL]
TC_ENGINES = [_lib.ENGINE_TCGEN05, _lib.ENGINE_TCGEN05_WIDE, _lib.ENGINE_TCGEN05_SWAP,
              _lib.ENGINE_TCGEN05_PAIR, _lib.ENGINE_TCGEN05_TALL]


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("shape,tokens", [(SMALL, 22), (SMALL, 300), (TINY, 16), (TINY, 512),
                                          (A, 1), (A, 8), (A, 64), (A, 640)])
def test_expert_engines_match_oracle(engine, shape, tokens):
    _expert_case(shape, tokens, engine, seed=100 + tokens)


@pytest.mark.parametrize("engine", TC_ENGINES)
def test_tcgen05_prefill_with_capacity_matches_oracle(engine):
    _expert_case(A, 2048, engine, seed=7, logits_kind="zipf",
                 capacity=wl.capacity_for(2048, A, 1.25))


@pytest.mark.parametrize("engine", TC_ENGINES)
@pytest.mark.parametrize("tokens,kind", [(1100, "uniform"), (2048, "zipf")])
def test_tcgen05_multi_chunk_experts_match_oracle(engine, tokens, kind):
    """Experts holding more than 256 rows: several row chunks (two-SM engine)
    or several 128-row tiles; Zipf without capacity piles thousands of rows
    onto the first experts."""
    _expert_case(SMALL, tokens, engine, seed=11 + tokens, logits_kind=kind)


@pytest.mark.parametrize("engine", [_lib.ENGINE_TCGEN05_WIDE, _lib.ENGINE_TCGEN05_SWAP])
@pytest.mark.parametrize("shape,tokens", [(SMALL, 300), (TINY, 16), (A, 8), (A, 640)])
def test_fused_row_gather_equals_packed_copy(engine, shape, tokens):
    """Token rows gathered by the GEMM's TMA loads (tile::gather4) give the
    same bits as the gate/up GEMM over a packed copy of the rows."""
    fused = _expert_case(shape, tokens, engine, seed=200 + tokens)
    packed = _expert_case(shape, tokens, engine, seed=200 + tokens, packed_rows=True)
    assert torch.equal(fused, packed)


@pytest.mark.parametrize("shape,tokens,kind", [
    (SMALL, 1100, "uniform"), (SMALL, 2048, "zipf"), (A, 2048, "zipf"), (A, 640, "uniform"),
    (wl.LayerShape("d-16", 4096, 1536, 16, 8), 640, "uniform"),
    (wl.LayerShape("d-32", 4096, 1536, 32, 8), 1100, "zipf")])
def test_tall_tiles_equal_wide_tiles_bit_for_bit(shape, tokens, kind):
    """256-row work items (two M=128 MMAs on one staged weight tile) compute
    every output element with the same K order as 128-row tiles: the same
    bits, for experts of every size (odd and even tile counts, remainders)."""
    tall = _expert_case(shape, tokens, _lib.ENGINE_TCGEN05_TALL, seed=40 + tokens,
                        logits_kind=kind)
    wide = _expert_case(shape, tokens, _lib.ENGINE_TCGEN05_WIDE, seed=40 + tokens,
                        logits_kind=kind, packed_rows=True)
    assert torch.equal(tall, wide)


@pytest.mark.parametrize("tokens,top_k,ep_size", [(1, 8, 2), (300, 8, 4), (4096, 8, 8),
                                                   (2500, 2, 16), (1030, 32, 3), (8192, 8, 8),
                                                   (512, 8, 8), (513, 8, 5)])
def test_ep_plan_slots_match_cpu_plan(tokens, top_k, ep_size):
    """Per-destination token and route slots (token order, route order) and
    the counts, against the CPU restatement; includes invalid ids."""
    from oracle.cpu_ops import CpuOps
    num_experts = 64
    gen = torch.Generator().manual_seed(tokens + ep_size)
    ids = torch.randint(-1, num_experts + 1, (tokens, top_k), generator=gen)
    owner = torch.randint(0, ep_size, (num_experts,), generator=gen).to(torch.int32)
    tok_d, rt_d, cnt_d = ops.ep_plan(ids.to(DEV), owner.to(DEV), ep_size, num_experts)
    tok_c, rt_c, cnt_c = CpuOps().ep_plan(ids, owner, ep_size, num_experts)
    torch.cuda.synchronize()
    assert torch.equal(tok_d.cpu(), tok_c)
    assert torch.equal(rt_d.cpu(), rt_c)
    assert torch.equal(cnt_d.cpu(), cnt_c)


def test_engines_agree_and_are_repeatable():
    outs = [_expert_case(A, 16, e, seed=3) for e in ENGINES]
    for other in outs[1:]:
        assert_close_rel(outs[0].float().cpu().numpy(), other.float().cpu().numpy())
    again = _expert_case(A, 16, _lib.ENGINE_TCGEN05, seed=3)
    assert torch.equal(again, outs[1])


def test_abi_errors_raise():
    logits = torch.zeros((4, 8), device=DEV)
    with pytest.raises(ValueError):
        ops.route_topk(logits, 9, True)
    with pytest.raises(NotImplementedError):
        ops.route_topk(torch.zeros((4, 2048), device=DEV), 8, True)
    assert pkg.device_status() == 0
