"""The 7B-class decode loop (decoder.py) and its glue kernels on the B200
against the CPU oracle (oracle/decoder_oracle.py, HF Llama semantics).

Glue kernels: RMSNorm and SwiGLU within one bf16 rounding of the oracle
(different rsqrt / exp implementations), rotary q within 2 bf16 ulps, the KV
bytes of the rotated k and of v exactly except where the two roundings land
on different sides of an fp8 tie.  Decoder: a 2-layer model with the 7B head
geometry stepped token by token from an empty cache; every step's logits
within 2e-2 of their maximum (north_star's fp32-accumulate bound), and the
greedy token equal wherever the oracle's top two logits are separated."""
import pytest
import torch

import decoder_oracle as DO

pytestmark = pytest.mark.gpu

TINY = dict(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, inter=1024, vocab=1000,
            rope_theta=1e6, eps=1e-5, block_size=16)


def _cfg(**kw):
    import decoder
    d = dict(TINY)
    d.update(kw)
    return decoder.DecoderConfig(**d)


def _bf16_ulps(a, b):
    """|a - b| in units of b's bf16 spacing."""
    spacing = torch.exp2(torch.floor(torch.log2(b.float().abs().clamp(min=1e-30))) - 7)
    return ((a.float() - b.float()).abs() / spacing)


def test_rmsnorm_residual(cuda):
    from _b200kv import check, lib
    g = torch.Generator().manual_seed(1)
    h = (3 * torch.randn(5, 4096, generator=g)).to(torch.bfloat16)
    dlt = torch.randn(5, 4096, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    hd, dd, wd = h.to(cuda), dlt.to(cuda), w.to(cuda)
    x = torch.empty_like(hd)
    st = torch.cuda.current_stream().cuda_stream
    check(lib.b200kv_rmsnorm_residual(hd.data_ptr(), dd.data_ptr(), wd.data_ptr(), x.data_ptr(),
                                      5, 4096, 1e-5, st), "rmsnorm")
    h2 = (h.float() + dlt.float()).to(torch.bfloat16)
    assert torch.equal(hd.cpu(), h2)
    want = DO.rmsnorm(h2, w, 1e-5)
    assert float(_bf16_ulps(x.cpu(), want).max()) <= 2.0
    # no residual
    check(lib.b200kv_rmsnorm_residual(hd.data_ptr(), None, wd.data_ptr(), x.data_ptr(), 5, 4096, 1e-5, st),
          "rmsnorm")
    assert torch.equal(hd.cpu(), h2)
    assert float(_bf16_ulps(x.cpu(), want).max()) <= 2.0


def test_swiglu(cuda):
    from _b200kv import check, lib
    g = torch.Generator().manual_seed(2)
    gu = (2 * torch.randn(3, 2 * 1536, generator=g)).to(torch.bfloat16)
    act = torch.empty(3, 1536, dtype=torch.bfloat16, device=cuda)
    gu_d = gu.to(cuda)
    check(lib.b200kv_swiglu(gu_d.data_ptr(), act.data_ptr(), 3, 1536,
                            torch.cuda.current_stream().cuda_stream), "swiglu")
    want = DO.swiglu(gu, 1536)
    assert float(_bf16_ulps(act.cpu(), want).max()) <= 2.0


def test_rope_kv_write(cuda):
    import decoder
    from _b200kv import KV_FP8_E4M3, check, lib
    hq, hkv, d, bs = 8, 2, 128, 16
    g = torch.Generator().manual_seed(3)
    T = 4
    qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    pos = torch.tensor([0, 5, 1000, 4095], dtype=torch.int32)
    slots = torch.tensor([3, 17, -1, 40], dtype=torch.int64)
    table = decoder.rope_table(4096, d, 1e6)
    assert torch.equal(table, DO.rope_table(4096, d, 1e6))
    kc = torch.zeros(4, bs, hkv, d, dtype=torch.uint8, device=cuda)
    vc = torch.zeros_like(kc)
    ks = torch.full((1,), 1 / 32, device=cuda)
    q = qkv.to(cuda)
    pos_d, table_d, slots_d = pos.to(cuda), table.to(cuda), slots.to(cuda)  # alive until the launch ran
    check(lib.b200kv_rope_kv_write(q.data_ptr(), q.stride(0), pos_d.data_ptr(),
                                   table_d.data_ptr(), 4096, slots_d.data_ptr(),
                                   kc.data_ptr(), vc.data_ptr(), *kc.stride()[:3], *vc.stride()[:3],
                                   ks.data_ptr(), ks.data_ptr(), T, hq, hkv, d, bs, KV_FP8_E4M3,
                                   torch.cuda.current_stream().cuda_stream), "rope_kv_write")
    qg, kcg, vcg = q.cpu().view(T, -1, d), kc.cpu(), vc.cpu()
    for t in range(T):
        heads = qkv[t].view(-1, d)
        want_q = DO.rope(heads[:hq], int(pos[t]), table)
        assert float(_bf16_ulps(qg[t, :hq], want_q).max()) <= 2.0
        assert torch.equal(qg[t, hq:], heads[hq:])  # k and v rows are left in place
        s = int(slots[t])
        if s < 0:
            continue
        k = DO.rope(heads[hq:hq + hkv], int(pos[t]), table)
        want_k = (k.float() * 32).to(torch.float8_e4m3fn).view(torch.uint8)
        want_v = (heads[hq + hkv:].float() * 32).to(torch.float8_e4m3fn).view(torch.uint8)
        got_k = kcg[s // bs, s % bs]
        assert (got_k.int() - want_k.int()).abs().max() <= 1  # adjacent codes at most
        assert float((got_k != want_k).float().mean()) < 0.02
        assert torch.equal(vcg[s // bs, s % bs], want_v)
    # nothing but the three valid slots was written (the -1 token is skipped)
    written = torch.zeros(4 * bs, dtype=torch.bool)
    written[[3, 17, 40]] = True
    assert int(kcg.view(4 * bs, -1)[~written].count_nonzero()) == 0
    assert int(vcg.view(4 * bs, -1)[~written].count_nonzero()) == 0


def _steps_match_oracle(cfg, cuda, batch, kernel, seed, max_ctx, steps):
    import decoder
    dec = decoder.MXFP4Decoder(cfg, cuda, batch, max_ctx, seed=seed, gen_device="cpu",
                               mxfp4_kernel=kernel)
    # the oracle's copy of the same weights (checkpoint scale layout [K/32, N])
    layers = []
    for li in range(cfg.layers):
        lay = decoder.random_layer(cfg, li, seed, "cpu")
        layers.append({k: ((v[0], v[1].t().contiguous()) if isinstance(v, tuple) else v)
                       for k, v in lay.items()})
    weights = dict(decoder.random_head(cfg, seed, "cpu"), layers=layers)
    nb = batch * dec.maxblk
    caches = [{"k": torch.zeros(nb, cfg.block_size, cfg.kv_heads, cfg.head_dim, dtype=torch.float8_e4m3fn),
               "v": torch.zeros(nb, cfg.block_size, cfg.kv_heads, cfg.head_dim, dtype=torch.float8_e4m3fn),
               "ks": 1 / 8, "vs": 1 / 8} for _ in range(cfg.layers)]
    table = DO.rope_table(max_ctx, cfg.head_dim, cfg.rope_theta)
    bt = dec.block_table.cpu()
    tokens = torch.tensor([3, 7, 11, 13][:batch], dtype=torch.int64)
    dec.tokens.copy_(tokens)
    positions = torch.zeros(batch, dtype=torch.int32)
    for step in range(steps):
        want = DO.decode_step(cfg, weights, caches, tokens, positions, bt, table)
        nxt = dec.step().cpu()
        got = dec.logits.cpu()
        err = (got - want).abs().max() / want.abs().max()
        print(f"step {step}: logits rel-to-max error {float(err):.4f}")
        assert float(err) < 2e-2, (step, float(err))
        top2 = want.topk(2, dim=1).values
        sep = (top2[:, 0] - top2[:, 1]) > 4 * float((got - want).abs().max())
        assert torch.equal(nxt[sep], want.argmax(1)[sep]), step
        tokens = nxt.clone()   # both continue from the GPU's tokens
        positions = positions + 1
    torch.cuda.synchronize()
    import _b200kv
    assert _b200kv.device_status() == 0


@pytest.mark.parametrize("batch,kernel", [(1, "auto"), (2, "auto"), (2, "mma.sync")])
def test_decoder_steps_match_oracle(cuda, batch, kernel):
    _steps_match_oracle(_cfg(), cuda, batch, kernel, seed=5, max_ctx=64, steps=6)


def test_decoder_7b_width_steps_match_oracle(cuda):
    """The 7B geometry config 4 times (hidden 4096, 32 q / 8 kv heads,
    intermediate 14336, vocab 128256, RoPE theta 1e6) with 2 of its 32 layers,
    batch 2, four decode steps: logits within 2e-2 of their maximum and greedy
    tokens equal where the oracle's top two are separated."""
    import dataclasses

    import decoder
    cfg = dataclasses.replace(decoder.SEVEN_B, layers=2)
    _steps_match_oracle(cfg, cuda, 2, "auto", seed=6, max_ctx=64, steps=4)


def test_decoder_step_in_cuda_graph(cuda):
    """Replaying a captured step continues the sequence exactly as eager steps."""
    import decoder
    cfg = _cfg()
    a = decoder.MXFP4Decoder(cfg, cuda, 2, 64, seed=9, gen_device="cpu")
    b = decoder.MXFP4Decoder(cfg, cuda, 2, 64, seed=9, gen_device="cpu")
    for dec in (a, b):
        dec.tokens.copy_(torch.tensor([1, 2]))
    toks_a = [a.step().clone() for _ in range(5)]
    first_b = b.step().clone()  # warm-up outside the capture (token 1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            b.step()
    torch.cuda.current_stream().wait_stream(s)
    # capturing does not run the step: b is still after one step
    toks_b = [first_b]
    for _ in range(4):
        graph.replay()
        torch.cuda.synchronize()
        toks_b.append(b.tokens.clone())
    for x, y in zip(toks_a, toks_b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("batch,P", [(1, 40), (3, 33)])
def test_decoder_prefill_then_decode_matches_oracle(cuda, batch, P):
    """prefill() (wide MXFP4 GEMMs at M = batch * P, RoPE + fp8 KV write of the
    prompt, varlen causal prefill attention) against the oracle stepping the
    prompt token by token: the last prompt token's logits within 2e-2 of their
    maximum, greedy tokens equal where separated; then three decode steps that
    read the cache the prefill wrote, same bounds.

    The weights use e8m0 scales 2^-10..2^-7. With the default 2^-8..2^-2 this
    random 2-layer model turns the last-ulp differences between the prefill
    and decode attention kernels (different key-block splits of the same
    softmax) into fp8 KV codes that differ in layer 1 and logits 5% apart,
    the GPU prefill against the GPU decode path alone; with the narrower
    scales the two GPU paths agree to 1e-3."""
    import decoder
    cfg = _cfg()
    seed, max_ctx = 8, 64
    scales = (117, 121)
    dec = decoder.MXFP4Decoder(cfg, cuda, batch, max_ctx, seed=seed, gen_device="cpu", scales=scales)
    layers = []
    for li in range(cfg.layers):
        lay = decoder.random_layer(cfg, li, seed, "cpu", scales)
        layers.append({k: ((v[0], v[1].t().contiguous()) if isinstance(v, tuple) else v) for k, v in lay.items()})
    weights = dict(decoder.random_head(cfg, seed, "cpu"), layers=layers)
    nb = batch * dec.maxblk
    caches = [{"k": torch.zeros(nb, cfg.block_size, cfg.kv_heads, cfg.head_dim, dtype=torch.float8_e4m3fn),
               "v": torch.zeros(nb, cfg.block_size, cfg.kv_heads, cfg.head_dim, dtype=torch.float8_e4m3fn),
               "ks": 1 / 8, "vs": 1 / 8} for _ in range(cfg.layers)]
    table = DO.rope_table(max_ctx, cfg.head_dim, cfg.rope_theta)
    bt = dec.block_table.cpu()
    prompts = torch.randint(0, cfg.vocab, (batch, P), generator=torch.Generator().manual_seed(P))
    for i in range(P):
        want = DO.decode_step(cfg, weights, caches, prompts[:, i], torch.full((batch,), i, dtype=torch.int32), bt,
                              table)
    nxt = dec.prefill(prompts.to(cuda)).cpu()
    positions = torch.full((batch,), P, dtype=torch.int32)
    for step in range(4):
        got = dec.logits.cpu()
        err = (got - want).abs().max() / want.abs().max()
        assert float(err) < 2e-2, (step, float(err))
        top2 = want.topk(2, dim=1).values
        sep = (top2[:, 0] - top2[:, 1]) > 4 * float((got - want).abs().max())
        assert torch.equal(nxt[sep], want.argmax(1)[sep]), step
        if step == 3:
            break
        tokens = nxt.clone()
        want = DO.decode_step(cfg, weights, caches, tokens, positions, bt, table)
        nxt = dec.step().cpu()
        positions = positions + 1
    torch.cuda.synchronize()
    import _b200kv
    assert _b200kv.device_status() == 0


def test_decoder_swiglu_epilogue_bit_equal_to_separate_kernel(cuda, monkeypatch):
    """gate_up with the SwiGLU epilogue (rows permuted at load time) against
    the same model with gate_up and the SwiGLU kernel as two launches: equal
    logits bit for bit through a prompt pass and decode steps (the prompt
    pass's wide GEMMs at K-split 1, the split the wide epilogue takes)."""
    import decoder
    monkeypatch.setenv("B200KV_GEMM_KSPLIT", "1")
    cfg = _cfg()
    a = decoder.MXFP4Decoder(cfg, cuda, 2, 64, seed=7, gen_device="cpu")
    b = decoder.MXFP4Decoder(cfg, cuda, 2, 64, seed=7, gen_device="cpu", fuse_swiglu=False)
    assert a.layers[0]["gate_up"][0] == "tcsw" and b.layers[0]["gate_up"][0] == "tc"
    prompts = torch.randint(0, cfg.vocab, (2, 20), generator=torch.Generator().manual_seed(1)).to(cuda)
    a.prefill(prompts)
    b.prefill(prompts)
    assert torch.equal(a.logits, b.logits)
    for _ in range(3):
        a.step()
        b.step()
        assert torch.equal(a.logits, b.logits)


def test_decode_step_prep(cuda):
    """b200kv_decode_step_prep: sequence lengths, KV slots through the block
    table and the embedding rows of the tokens, against torch."""
    from _b200kv import check, lib
    g = torch.Generator().manual_seed(21)
    B, H, V, bs = 5, 512, 300, 16
    embed = torch.randn(V, H, generator=g).to(torch.bfloat16).to(cuda)
    tokens = torch.randint(0, V, (B,), generator=g).to(cuda)
    pos = torch.tensor([0, 15, 16, 1000, 63], dtype=torch.int32, device=cuda)
    bt = torch.randperm(5 * 64, generator=g).to(torch.int32).view(5, 64).to(cuda)
    seq_lens = torch.zeros(B, dtype=torch.int32, device=cuda)
    slots = torch.zeros(B, dtype=torch.int64, device=cuda)
    h = torch.zeros(B, H, dtype=torch.bfloat16, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    check(lib.b200kv_decode_step_prep(pos.data_ptr(), tokens.data_ptr(), embed.data_ptr(), H, V, bt.data_ptr(),
                                      bt.stride(0), bt.shape[1], bs, B, seq_lens.data_ptr(), slots.data_ptr(),
                                      h.data_ptr(), st), "b200kv_decode_step_prep")
    torch.cuda.synchronize()
    assert torch.equal(seq_lens, pos + 1)
    want = bt.gather(1, (pos // bs).long().unsqueeze(1)).squeeze(1).long() * bs + (pos % bs).long()
    assert torch.equal(slots, want)
    assert torch.equal(h, embed[tokens])
    import _b200kv
    assert _b200kv.device_status() == 0
    # an id past the vocabulary and a position past the row: nothing read out
    # of the tables, a zero row, slot -1 and the index-range status
    tokens[1] = V
    pos[3] = 64 * bs
    check(lib.b200kv_decode_step_prep(pos.data_ptr(), tokens.data_ptr(), embed.data_ptr(), H, V, bt.data_ptr(),
                                      bt.stride(0), bt.shape[1], bs, B, seq_lens.data_ptr(), slots.data_ptr(),
                                      h.data_ptr(), st), "b200kv_decode_step_prep")
    torch.cuda.synchronize()
    assert torch.all(h[1] == 0) and int(slots[3]) == -1
    assert torch.equal(h[0], embed[tokens[0]]) and int(slots[0]) == int(want[0])
    assert _b200kv.device_status() == 0x105
    _b200kv.reset_device_status()
