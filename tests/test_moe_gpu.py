"""gpt-oss MoE on the B200: router top-k, permute, MXFP4 grouped GEMMs and
un-permute against the CPU oracle / plain torch, then a whole gpt-oss-style
decode (sinks, sliding window, YaRN, MXFP4 experts) against the oracle.

Router logits are the bf16 values nearest to the exact x . w + b (rounded
once, ties to even), so they do not depend on summation order: the kernel's
logits, top-k indices and softmax weights must equal the oracle's bit for
bit, with zero tolerance, on every token, including inputs that leave the
kernel's fast fixed-point window (subnormals, wide exponent spreads)."""
import pytest
import torch

from oracle import decode_ref as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from fluidgpu_b200 import build

    build.build()
    yield
    from fluidgpu_b200 import kernels

    kernels.check_device("moe tests")


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _router_case(T, H, E, k, kind, g):
    x = torch.randn(T, H, generator=g)
    w = torch.randn(E, H, generator=g) * 0.05
    b = torch.randn(E, generator=g) * 0.1
    if kind == "wide":
        # exponent spreads beyond the fast window, subnormal inputs, zero rows
        x[0, ::7] *= 2.0 ** -60
        x[1, 3] = 2.0 ** -130
        w[1, ::5] *= 2.0 ** 40
        x[2] = 0.0
    elif kind == "ties":
        # small integers: many logits tie exactly, and many sums land on
        # bf16 midpoints
        x = torch.randint(-3, 4, (T, H), generator=g).float()
        w = torch.randint(-2, 3, (E, H), generator=g).float() / 4
        b = torch.zeros(E)
    return x.to(torch.bfloat16), w.to(torch.bfloat16), b.to(torch.bfloat16)


@pytest.mark.parametrize("T,H,E,k,kind", [(128, 2880, 32, 4, "normal"), (7, 256, 8, 2, "normal"),
                                          (64, 512, 64, 8, "normal"), (1, 64, 4, 1, "normal"),
                                          (16, 1024, 32, 4, "wide"), (32, 512, 32, 4, "ties")])
def test_router_topk_exact(T, H, E, k, kind):
    from fluidgpu_b200 import moe

    x, w, b = _router_case(T, H, E, k, kind, _g(1))
    wts, idx, lg = moe.router_topk(x.to(DEV), w.to(DEV), b.to(DEV), k, logits=True)
    exp_w, exp_i, exp_lg = ref.router_topk_exact(x, w, b, k)
    assert torch.equal(lg.cpu().view(torch.int16), exp_lg.view(torch.int16)), "router logits"
    assert torch.equal(idx.cpu().long(), exp_i), "router indices"
    assert torch.equal(wts.cpu().view(torch.int16), exp_w.view(torch.int16)), "router weights"
    if kind == "normal":
        # and the bf16 linear of the reference differs by at most one bf16
        # step where its accumulation rounded
        lin = torch.nn.functional.linear(x, w, b).float()
        step = 2.0 ** (torch.floor(torch.log2(lin.abs().clamp(min=2.0 ** -126))) - 7)
        assert ((lg.cpu().float() - lin).abs() <= step).all()


def test_topk_softmax_given_logits_exact():
    from fluidgpu_b200.vllm_ops import topk_softmax

    g = _g(7)
    lg = (torch.randn(37, 32, generator=g) * 2).to(torch.bfloat16)
    lg[5, 3] = lg[5, 9]  # a tie: the lower id first
    wts, idx = topk_softmax(lg.to(DEV), 4)
    top_v, top_i = ref.topk_lowest(lg.float(), 4)
    assert torch.equal(idx.cpu().long(), top_i)
    assert torch.equal(wts.cpu().view(torch.int16), ref.softmax_topk_bf16(top_v).view(torch.int16))


@pytest.mark.parametrize("T,k,E", [(128, 4, 32), (5, 2, 8), (300, 4, 32), (64, 8, 64)])
def test_permute_exact(T, k, E):
    from fluidgpu_b200 import moe

    g = _g(2)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    if T > 100:
        idx[: T // 2, 0] = 3  # a hot expert: several token tiles
    r = moe.Routing(idx.to(DEV), E)
    flat = idx.reshape(-1).long()
    counts = torch.bincount(flat, minlength=E)
    offsets = torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)])
    assert torch.equal(r.offsets.cpu().long(), offsets)
    exp_perm = torch.argsort(flat * (T * k) + torch.arange(T * k), stable=True)
    assert torch.equal(r.perm_pair.cpu().long(), exp_perm)
    inv = torch.empty_like(exp_perm)
    inv[exp_perm] = torch.arange(T * k)
    assert torch.equal(r.inv.cpu().long(), inv)
    items = [(e, t) for e in range(E) for t in range((int(counts[e]) + r.BN - 1) // r.BN)]
    n = int(r.item_count.item())
    assert n == len(items)
    assert r.items.cpu().view(-1, 2)[:n].tolist() == [list(x) for x in items]


def _ref_expert_gemm(x_perm, deq_w, bias, offsets, epilogue):
    """fp32 reference of the grouped GEMM on the dequantised (exact bf16) weights."""
    out = []
    for e in range(deq_w.shape[0]):
        xs = x_perm[offsets[e]:offsets[e + 1]].float()
        y = xs @ deq_w[e].float().T + bias[e].float()
        if epilogue == "swiglu_oai":
            y = y.to(torch.bfloat16).float()
            I = y.shape[1] // 2
            g, u = y.view(-1, I // 64, 2, 64)[:, :, 0].reshape(-1, I), y.view(-1, I // 64, 2, 64)[:, :, 1].reshape(-1, I)
            y = ref.swiglu_oai(g.to(torch.bfloat16), u.to(torch.bfloat16)).float()
        out.append(y)
    return torch.cat(out)


@pytest.mark.parametrize("T,k,E,H,I", [(128, 4, 32, 2880, 2880), (9, 2, 8, 256, 512), (40, 4, 16, 512, 256)])
def test_grouped_mxfp4_gemms(T, k, E, H, I):
    from fluidgpu_b200 import _lib, moe

    g = _g(3)
    w1 = torch.randn(E, 2 * I, H, generator=g) * 0.02      # already 64-interleaved order here
    w2 = torch.randn(E, H, I, generator=g) * 0.02
    b1 = (torch.randn(E, 2 * I, generator=g) * 0.1).to(torch.bfloat16)
    b2 = (torch.randn(E, H, generator=g) * 0.1).to(torch.bfloat16)
    v1, s1 = moe.quantize_mxfp4(w1.to(DEV))
    v2, s2 = moe.quantize_mxfp4(w2.to(DEV))
    d1 = moe.dequantize_mxfp4(v1, s1).cpu()
    d2 = moe.dequantize_mxfp4(v2, s2).cpu()
    # the product quantiser agrees with the oracle's restatement
    ov, os_ = ref.mxfp4_quantize(w1[:2, :128])
    assert torch.equal(ref.mxfp4_dequantize(ov, os_), d1[:2, :128])
    p1, p2 = moe.pack_mxfp4(v1, s1), moe.pack_mxfp4(v2, s2)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    r = moe.Routing(idx.to(DEV), E)
    x_perm = x[r.perm_pair.cpu().long() // k]
    offsets = r.offsets.cpu().tolist()
    act = moe.grouped_gemm(x_perm.to(DEV, torch.float16).contiguous(), p1, b1.to(DEV), r, 2 * I, H,
                           _lib.FG_EPI_SWIGLU_OAI)
    assert act.dtype == torch.float16
    exp_act = _ref_expert_gemm(x_perm, d1, b1, offsets, "swiglu_oai")
    err = (act.cpu().float() - exp_act).abs().max().item()
    assert err <= 2e-2 * exp_act.abs().max().item() + 1e-3, err
    y = moe.grouped_gemm(act, p2, b2.to(DEV), r, H, I, _lib.FG_EPI_STORE)
    exp_y = _ref_expert_gemm(act.cpu(), d2, b2, offsets, "store")
    err = (y.cpu().float() - exp_y).abs().max().item()
    assert err <= 1e-2 * exp_y.abs().max().item() + 1e-3, err


def test_unpermute_order_and_residual():
    from fluidgpu_b200 import _lib, moe

    g = _g(4)
    T, k, E, H = 33, 4, 16, 256
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    wts = torch.softmax(torch.randn(T, k, generator=g), -1).to(torch.bfloat16)
    r = moe.Routing(idx.to(DEV), E)
    y = torch.randn(T * k, H, generator=g).to(torch.bfloat16)
    res = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    yd, idxd, wd, rd = y.to(DEV), idx.to(DEV), wts.to(DEV), res.to(DEV)  # keep the device copies alive
    _lib.call("fg_moe_unpermute", yd.data_ptr(), r.inv.data_ptr(), idxd.data_ptr(), wd.data_ptr(),
              rd.data_ptr(), out.data_ptr(), T, k, H, 0, E, 0, torch.cuda.current_stream().cuda_stream)
    inv = r.inv.cpu().long()
    exp = torch.zeros(T, H, dtype=torch.bfloat16)
    for t in range(T):
        for j in sorted(range(k), key=lambda j: int(idx[t, j])):  # index_add_ order: ascending expert
            exp[t] += y[inv[t * k + j]] * wts[t, j]
    exp = res + exp
    assert torch.equal(out.cpu(), exp)
    # expert-parallel halves: each shard's slots only, fp32 partials; their
    # sum is the shard-ordered sum of the two bf16 partial sums
    parts = torch.empty(2, T, H, dtype=torch.float32, device=DEV)
    for sh, (lo, hi) in enumerate(((0, E // 2), (E // 2, E))):
        _lib.call("fg_moe_unpermute", yd.data_ptr(), r.inv.data_ptr(), idxd.data_ptr(), wd.data_ptr(), None,
                  parts[sh].data_ptr(), T, k, H, lo, hi, 1, torch.cuda.current_stream().cuda_stream)
        ref = torch.zeros(T, H, dtype=torch.bfloat16)
        for t in range(T):
            for j in sorted(range(k), key=lambda j: int(idx[t, j])):
                if lo <= int(idx[t, j]) < hi:
                    ref[t] += y[inv[t * k + j]] * wts[t, j]
        assert torch.equal(parts[sh].cpu(), ref.float()), f"shard {sh} partial"
    from fluidgpu_b200 import kernels

    total = kernels.sum_partials(parts)
    assert torch.equal(total.cpu(), (parts[0].cpu() + parts[1].cpu()).to(torch.bfloat16))


def _tiny_gptoss(seed=0):
    from transformers.models.gpt_oss import GptOssConfig, GptOssForCausalLM

    from fluidgpu_b200 import moe

    torch.manual_seed(seed)
    cfg = GptOssConfig(num_hidden_layers=2, num_local_experts=8, vocab_size=1024, hidden_size=512,
                       intermediate_size=256, head_dim=64, num_attention_heads=8, num_key_value_heads=2,
                       sliding_window=16, num_experts_per_tok=2,
                       layer_types=["sliding_attention", "full_attention"], max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    model = GptOssForCausalLM(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            ex = layer.mlp.experts
            # make the experts MXFP4-exact (a real gpt-oss checkpoint is MXFP4)
            for name in ("gate_up_proj", "down_proj"):
                p = getattr(ex, name)
                wt = p.data.transpose(1, 2).float()
                v, s = moe.quantize_mxfp4(wt)
                p.data.copy_(moe.dequantize_mxfp4(v, s).transpose(1, 2).to(p.dtype))
            layer.mlp.router.weight.data.normal_(0, 0.2)  # spread router logits
            layer.self_attn.sinks.data.normal_(0, 1.0)
    return model


def test_gpt_oss_decode_matches_oracle():
    from fluidgpu_b200 import kernels
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights

    model = _tiny_gptoss()
    w = ModelWeights.from_hf(model, DEV)
    batch, prompt, steps = 4, 20, 12
    eng = DecodeEngine(w, EngineConfig(model_name="tiny-gpt-oss", max_seq_len=64, world_size=1,
                                       device="cuda:0", max_batch=batch))
    eng.runner.record_routing = True
    spec = ref.spec_from_hf(model.config)
    Wl = {i: (w.layers[i]["router_w"].cpu(), w.layers[i]["router_b"].cpu()) for i in range(spec.num_layers)}
    wo = ref.weights_from_hf(model)
    truth = ref.OracleModel(spec, {k: v.float() for k, v in wo.items()}, torch.float32)
    bf16 = ref.OracleModel(spec, wo, torch.bfloat16)
    g = _g(5)
    prompts = torch.randint(0, 1024, (batch, prompt), generator=g)
    eng.start(batch, reserve_tokens=prompt + steps + 2)
    truth.reset(batch)
    bf16.reset(batch)
    checked = 0
    # every step within atol/rtol of the fp32 or of the bf16 oracle, else the
    # run's worst deviation within 1.25x the bf16 oracle's worst (one step's
    # maximum over a vocabulary row is noisy; the bf16 oracle also varies a
    # little with the host's CPU matmul kernels)
    worst, ref_worst, loose = 0.0, 0.0, []
    for t in range(prompt + steps):
        tok = prompts[:, t] if t < prompt else ref.argmax_lowest(lt.float())
        got = eng.runner.decode_step(tok.to(DEV)).reshape(batch, -1).float().cpu()
        lt = truth.step(tok)
        lb = bf16.step(tok)
        err = (got - lt).abs()
        worst = max(worst, err.max().item())
        ref_worst = max(ref_worst, (lb.float() - lt).abs().max().item())
        near_truth = bool((err <= 2e-2 + 1e-2 * lt.abs()).all())
        near_bf16 = bool(((got - lb.float()).abs() <= 2e-2 + 1e-2 * lb.float().abs()).all())
        if not (near_truth or near_bf16):
            loose.append(t)
        # router: on the rows the GPU router saw, its expert ids equal the
        # oracle router's exactly, in order, for every token and layer
        for layer in range(spec.num_layers):
            gi = eng.runner.last_routing[layer].cpu().long()
            _, oi, _ = ref.router_topk_exact(eng.runner.last_router_input[layer].cpu(), *Wl[layer], spec.top_k)
            assert torch.equal(gi, oi), f"step {t} layer {layer}: router indices differ"
            checked += gi.shape[0]
    assert not loose or worst <= 1.25 * ref_worst + 1e-3, (loose, worst, ref_worst)
    assert checked == batch * (prompt + steps) * spec.num_layers
    kernels.check_device("gpt-oss decode")


def test_mxfp4_scale_window():
    """Rows whose block scales spread over up to 36 binades (and all-zero
    blocks with arbitrary scales) give the exact dequantised products; a
    nonzero block further below its row's largest is refused at packing."""
    from fluidgpu_b200 import _lib, kernels, moe

    g = _g(6)
    E, N, K, T, k = 2, 128, 256, 8, 1
    v = torch.randint(0, 256, (E, N, K // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    s = torch.full((E, N, K // 32), 120, dtype=torch.uint8)
    s[:, :, 1] = 120 + 13        # largest block of the row
    s[:, :, 2] = 120 + 13 - 36   # lowest exact block
    s[:, 5, 3] = 250             # an all-zero block with a huge scale does not count
    v[:, 5, 48:64] = 0
    p = moe.pack_mxfp4(v.to(DEV), s.to(DEV))
    kernels.check_device("in-window packing")
    w = moe.dequantize_mxfp4(v, s, torch.float32)
    idx = torch.zeros((T, k), dtype=torch.int32)
    idx[T // 2:] = 1
    r = moe.Routing(idx.to(DEV), E)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    x_perm = x[r.perm_pair.cpu().long() // k]
    y = moe.grouped_gemm(x_perm.to(DEV, torch.float16).contiguous(), p, None, r, N, K,
                         _lib.FG_EPI_STORE).cpu().float()
    offs = r.offsets.cpu().tolist()
    ref = torch.cat([x_perm[offs[e]:offs[e + 1]].double() @ w[e].double().T for e in range(E)])
    ref = ref.float()
    assert torch.allclose(y, ref, rtol=2 ** -7, atol=1e-4 * ref.abs().max().item()), (y - ref).abs().max()
    s[0, 7, 4] = 120 + 13 - 37   # one binade too far, with nonzero values
    v[0, 7, 64:80] = 0x11
    moe.pack_mxfp4(v.to(DEV), s.to(DEV))
    with pytest.raises(RuntimeError, match="MXFP4 block scale"):
        kernels.check_device("out-of-window packing")
