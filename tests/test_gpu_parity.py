"""GPU parity: libotq through its C ABI against the reference's own vectors
(tests/golden/reference_vectors.npz, made by running the reference) and against the CPU
oracle on seeded inputs. Integer and byte results and the MM outputs are compared bit for bit;
the weight-only 4-bit layer within a stated float tolerance."""
import hashlib

import numpy as np
import pytest

from conftest import bits, rel
from oracle import fp32 as F
from oracle import mx as X
from oracle import survey as SV
from opentpu_b200 import workloads as WL

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FMT_OF_WF = {0: "int8", 1: "int4", 2: "fp4", 3: "nvfp4"}
# weight-only 4-bit: fp32 accumulation against float64, relative to max |y|
G32_TOL = 2e-6


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    from opentpu_b200 import linear
    return linear


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ---------------------------------------------------------------------------- QACT
@pytest.mark.parametrize("g", [32, 128])
@pytest.mark.parametrize("row", [0, 1])
def test_qact_matches_reference(ops, golden, g, row):
    q, S, d = ops.quantize_act(dev(golden["qact_x"]), row_mode=bool(row), group=g)
    assert np.array_equal(host(q), golden[f"qact_g{g}_r{row}_q"])
    assert np.array_equal(bits(host(S)), golden[f"qact_g{g}_r{row}_S"])
    if not row:
        assert np.array_equal(host(d), golden[f"qact_g{g}_r{row}_d"])


# ---------------------------------------------------------------------------- weight formats
@pytest.mark.parametrize("fmt", X.FORMATS)
def test_weight_quantizers_match_reference(ops, golden, fmt):
    W = golden["fmt_W"]
    w = ops.PackedWeight.from_float(dev(W), fmt)
    rows, srows = host(w.rows), host(w.srows)
    want_r, want_s = golden[f"fmt_{fmt}_rows"], golden[f"fmt_{fmt}_srows"]
    assert np.array_equal(rows[:, :want_r.shape[1]], want_r)
    assert np.array_equal(srows, want_s)


def test_rsc_rows_match_reference(ops, golden):
    w = ops.PackedWeight.from_float(dev(golden["fmt_W"]), "int8-row")
    assert np.array_equal(host(w.rows)[:, :1024].view(np.int8), golden["fmt_rsc_q"])
    assert np.array_equal(host(w.srows), golden["fmt_rsc_s"])


# ---------------------------------------------------------------------------- MM programs
def _mm_case(golden, key):
    wf, unit, rsc, k0, KB, M, N, row_mode = (int(v) for v in golden[key + "_meta"])
    return FMT_OF_WF[wf], bool(unit), bool(rsc), k0, KB, M, N, bool(row_mode)


def _packed(ops, golden, key, fmt, unit, rsc, k0, K):
    srows = None if unit else golden[key + "_srows"]
    return ops.PackedWeight.from_packed(golden[key + "_data"], srows, fmt, K, k0=k0, rsc=rsc)


@pytest.mark.parametrize("path", ["mm", "qmm"])
def test_mm_programs_match_reference(ops, golden, path):
    """Every format x UNIT / RSC / k0 / ROW case the reference ISA simulator ran at D=128:
    MM of the simulator's own ACT bytes (path mm) and QACT+MM fused from fp32 (path qmm)."""
    for key in [str(k) for k in golden["mm128_cases"]]:
        fmt, unit, rsc, k0, KB, M, N, row_mode = _mm_case(golden, key)
        K = KB * 128
        w = _packed(ops, golden, key, fmt, unit, rsc, k0, K)
        if path == "mm":
            q = dev(golden[key + "_q"])
            Sa = dev(golden[key + "_Sa"].view(np.float32))
            da = dev(golden[key + "_da"].reshape(M, KB * 4))
            y = ops.mm(q, Sa, da, w)
        else:
            y = ops.qlinear(dev(golden[key + "_x"]), w, row_mode=row_mode)
        assert np.array_equal(bits(host(y)), golden[key + "_y"]), (key, fmt, unit, rsc, k0)


def test_acc_and_ascale_match_reference(ops, golden):
    k = "mm128_acc"
    x, data, srows = golden[k + "_x"], golden[k + "_data"], golden[k + "_srows"]
    K = x.shape[1]
    w = ops.PackedWeight.from_packed(data, srows, "int8", K)
    out = dev(golden[k + "_old"])
    ops.qlinear(dev(x), w, out=out, acc=True)
    assert np.array_equal(bits(host(out)), golden[k + "_y_acc"])
    wu = ops.PackedWeight.from_packed(data, None, "int8", K)
    out = dev(golden[k + "_old"])
    ops.qlinear(dev(x), wu, out=out, alpha=dev(golden[k + "_alpha"]))
    assert np.array_equal(bits(host(out)), golden[k + "_y_ascale"])


@pytest.mark.parametrize("fmt", X.FORMATS)
def test_k_dot_pipeline_matches_reference(ops, golden, fmt):
    """runtime.launch(k_dot): quantize the weight on the GPU, QACT + MM on the GPU."""
    x, W = golden[f"dot_{fmt}_x"], golden[f"dot_{fmt}_W"]
    w = ops.PackedWeight.from_float(dev(W), fmt)
    y = ops.qlinear(dev(x), w)
    assert np.array_equal(bits(host(y)), golden[f"dot_{fmt}_y"])


def test_config1_matches_reference(ops, golden):
    W, x = WL.gemv_config1(0)
    w = ops.PackedWeight.from_float(dev(W), "int8-row")
    r, s = host(w.rows)[:, :1024], host(w.srows)
    assert hashlib.sha256(r.tobytes() + s.tobytes()).hexdigest() == str(golden["cfg1_rsc_digest"])
    y = ops.qlinear(dev(x), w)
    assert np.array_equal(bits(host(y)), golden["cfg1_rsc_y"])
    w8 = ops.PackedWeight.from_float(dev(W), "int8")
    r, s = host(w8.rows)[:, :1024], host(w8.srows)
    assert hashlib.sha256(r.tobytes() + s.tobytes()).hexdigest() == \
        str(golden["cfg1_int8x_digest"])
    assert np.array_equal(bits(host(ops.qlinear(dev(x), w8))), golden["cfg1_int8x_y"])


# ---------------------------------------------------------------------------- vs the oracle
# every work decomposition of the GEMV (0: the pick; 32: 32-row blocks; 1: 8-row blocks;
# 2, 4, 8: 8-row blocks with K split over that many warps)
SPLITS = (0, 1, 2, 4, 8, 32)
SHAPES = [(1, 1, 128), (1, 5, 256), (3, 37, 384), (1, 1024, 1024), (8, 513, 1024),
          (2, 300, 3072), (4, 64, 11008), (5, 2048, 2048), (1, 7, 32640)]


@pytest.mark.parametrize("fmt", ["int8", "int8-row", "int4", "fp4", "nvfp4"])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_qlinear_matches_oracle(ops, fmt, M, N, K):
    rng = np.random.default_rng(M * 1000003 + N * 131 + K)
    if fmt == "nvfp4" and K == 32640:
        K = 32512
    W = WL.spread_rows(rng, N, K, 2.0, 32)
    x = WL.spread_acts(rng, M, K, 3.0, 8)
    w = ops.PackedWeight.from_float(dev(W), fmt)
    mfmt = "int8" if fmt == "int8-row" else fmt
    rows, srows = host(w.rows), host(w.srows)
    if fmt == "int8-row":
        want_rows, want_srows = X.quantize_rows_rsc(W)
    else:
        want_rows, want_srows = X.quantize_weights(W, fmt)
    assert np.array_equal(rows[:, :want_rows.shape[1]], want_rows)
    assert np.array_equal(srows, want_srows)
    want = X.qlinear(x, want_rows, want_srows, mfmt, rsc=fmt == "int8-row")
    for split in SPLITS:
        y = ops.qlinear(dev(x), w, k_split=split, pdl=split >= 2)
        assert np.array_equal(bits(host(y)), bits(want)), (fmt, M, N, K, split)
    from opentpu_b200 import _lib
    assert _lib.status_word() == 0
    q, S, d = ops.quantize_act(dev(x))
    qo, So, do = F.quantize_rows(x, 32)
    assert np.array_equal(host(q), qo) and np.array_equal(bits(host(S)), bits(So))
    assert np.array_equal(host(d), do)
    assert np.array_equal(bits(host(ops.mm(q, S, d, w))), bits(want))


def test_row_mode_and_k0_column_part(ops):
    rng = np.random.default_rng(9)
    N, K = 96, 1024
    W = WL.spread_rows(rng, N, K, 2.0, 32)
    x = WL.spread_acts(rng, 2, 512, 2.0, 8)
    rows, srows = X.quantize_weights(W, "int4")
    part = rows[:, 128:384]                         # columns 256..768: blocks 2..5
    w = ops.PackedWeight.from_packed(part, srows, "int4", 512, k0=2)
    want = X.qlinear(x, part, srows, "int4", k0=2, row_mode=True)
    assert np.array_equal(bits(host(ops.qlinear(dev(x), w, row_mode=True))), bits(want))


@pytest.mark.parametrize("fmt", ["int8-row", "int4"])
def test_lm_head_full_size(ops, fmt):
    """The LM head of the Qwen3-0.6B shape (151936 x 1024) at M = 1 and 8, every engine."""
    rng = np.random.default_rng(0)
    N, K = WL.QWEN3_0_6B.vocab, WL.QWEN3_0_6B.hidden
    Wt = torch.randn(N, K, generator=torch.Generator().manual_seed(0)) * 0.02
    x = rng.standard_normal((8, K)).astype(np.float32)
    w = ops.PackedWeight.from_float(Wt.cuda(), fmt)
    rows, srows = host(w.rows), host(w.srows)
    want = X.qlinear(x, rows, srows, "int8" if fmt == "int8-row" else fmt,
                     rsc=fmt == "int8-row")
    for split in SPLITS:
        y1 = ops.qlinear(dev(x[:1]), w, k_split=split)
        assert np.array_equal(bits(host(y1)), bits(want[:1])), split
        y8 = ops.qlinear(dev(x), w, k_split=split)
        assert np.array_equal(bits(host(y8)), bits(want)), split


def test_errors_are_refused_on_the_host(ops):
    w = ops.PackedWeight.from_float(torch.randn(64, 256, device="cuda"), "int8")
    with pytest.raises(ValueError):
        ops.qlinear(torch.randn(3, 128, device="cuda"), w)          # K mismatch
    bad = ops.PackedWeight("nvfp4", 64, 256, w.rows, w.srows[:, :4])
    with pytest.raises(ValueError):
        ops.qlinear(torch.randn(1, 256, device="cuda"), bad)        # scale rows too short
    with pytest.raises(ValueError):
        ops.PackedWeight.from_float(torch.randn(8, 100, device="cuda"), "int8")   # K % 128


# ---------------------------------------------------------------------------- int4-g32
def test_g32_quantizer_matches_reference(ops, golden):
    w = ops.PackedWeight.from_float(dev(golden["g32_W"]), "int4-g32")
    codes = SV.unpack_g32(host(w.rows), 512).astype(np.float64)
    scales = host(w.srows).astype(np.float64)
    assert np.array_equal(scales, golden["g32_scales"])
    deq = (codes.reshape(40, 16, 32) * scales[..., None]).reshape(40, 512).astype(np.float32)
    assert np.array_equal(deq, golden["g32_deq"])


@pytest.mark.parametrize("M,N,K", [(1, 1024, 1024), (4, 3072, 1024), (1, 1024, 3072),
                                   (8, 640, 8192), (2, 100, 11008), (1, 151936, 1024),
                                   (1, 1000, 4096), (1, 37, 11008)])
def test_g32_linear_within_tolerance(ops, M, N, K):
    rng = np.random.default_rng(N + K + M)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = ops.PackedWeight.from_float(dev(W), "int4-g32")
    codes, scales, _ = SV.quantize_g32(W)
    assert np.array_equal(SV.unpack_g32(host(w.rows), K), codes)
    want = SV.linear_g32(x, codes, scales)
    got = host(ops.qlinear(dev(x), w)).astype(np.float64)
    assert np.abs(got - want).max() <= G32_TOL * np.abs(want).max()
    assert rel(got, want) < G32_TOL


# ---------------------------------------------------------------------------- chains
def test_chain_matches_oracle(ops):
    """otq_qmm_chain: projections of several formats in one call (one launch per run of a
    format), each reading an earlier projection's output, one with ACC, a tall one taking the
    32-row blocks: bit-exact with the oracle run in the same order."""
    from opentpu_b200 import _lib
    rng = np.random.default_rng(5)
    # (format, N, K, acc); projection i reads the first K outputs of projection i - 1
    specs = [("int8-row", 640, 256, False), ("int8-row", 40064, 512, False),
             ("int8", 300, 1024, False), ("int4", 512, 256, False),
             ("int8-row", 2048, 384, True), ("nvfp4", 130, 128, False), ("fp4", 256, 128, False)]
    x0 = WL.spread_acts(rng, 1, specs[0][2], 3.0, 8)[0]
    ws, outs, steps, host_w = [], [], [], []
    prev = torch.tensor(x0, device="cuda")
    olds = []
    for i, (fmt, N, K, acc) in enumerate(specs):
        W = WL.spread_rows(rng, N, K, 2.0, 32)
        w = ops.PackedWeight.from_float(dev(W), fmt)
        y = torch.tensor(rng.standard_normal(N).astype(np.float32), device="cuda")
        olds.append(host(y).copy())
        x = prev[:K]
        steps.append((x, w, y, acc, False))
        ws.append(w)
        outs.append(y)
        host_w.append((host(w.rows), host(w.srows), fmt))
        prev = y
    table = ops.chain_table(steps)
    ops.qlinear_chain(table)
    torch.cuda.synchronize()
    assert _lib.status_word() == 0
    xin = x0
    for (fmt, N, K, acc), (rows, srows, f), y, old in zip(specs, host_w, outs, olds):
        mfmt = "int8" if f == "int8-row" else f
        want = X.qlinear(xin[None, :K], rows, srows, mfmt, rsc=f == "int8-row")[0]
        if acc:
            want = F.fadd(old, want)
        got = host(y)
        assert np.array_equal(bits(got), bits(want)), (fmt, N, K)
        xin = got
    # the same table again gives the same bits (the grid barrier re-arms itself)
    before = [host(y).copy() for y in outs]
    for (x, w, y, acc, rm), old in zip(steps, olds):
        y.copy_(torch.tensor(old, device="cuda"))
    ops.qlinear_chain(table)
    torch.cuda.synchronize()
    assert all(np.array_equal(bits(host(y)), bits(b)) for y, b in zip(outs, before))


def test_decode_chain_chained_equals_launch_per_projection():
    from opentpu_b200.decode import DecodeChain
    a = DecodeChain(WL.TINY, chained=True)
    b = DecodeChain(WL.TINY, chained=False)
    assert a.launches == 2 and b.launches == len(b.plan) + 1   # + the argmax launch
    a.step_eager()
    b.step_eager()
    torch.cuda.synchronize()
    for i in range(len(a.plan)):
        assert np.array_equal(bits(host(a.full_out(i))), bits(host(b.full_out(i))))
    a.capture()
    a.replay(3)
    torch.cuda.synchronize()
    assert np.array_equal(bits(host(a.logits())), bits(host(b.logits())))
    b.capture()
    b.replay(1)
    torch.cuda.synchronize()
    assert int(a.token[0]) == int(b.token[0])


# ---------------------------------------------------------------------------- token level
def _token_parity(dev_tokens, dev_logits, ora, prompt):
    """The reference's rule for a greedy run against a golden (tests/test_validate.py:124-164
    _top1_where_clear), teacher forced on the device's tokens: at every step whose golden top-1
    leads its runner-up by more than the golden's own noise floor (the largest logit change
    1-ulp input noise causes, tools/validate.py Golden._noisy; a fixed threshold, not the run's
    own error), the device's token is the golden's first maximal logit. The device's logits
    must also follow the golden's: their smallest per-step cosine to the golden departs from 1
    by at most twice as much as the 1-ulp noise run's does, or 2e-4, whichever is larger (on a
    small model the noise run may flip no quantization at all). Returns (clear steps, floor)."""
    from oracle.model import clear_steps, noise_run
    ref = ora.forced(prompt, dev_tokens)
    floor, noise_cos = noise_run(ora, prompt, dev_tokens, ref)
    clear = clear_steps(ref, floor)
    cos = [float(np.dot(a, b) / np.linalg.norm(a) / np.linalg.norm(b))
           for a, b in zip(dev_logits.astype(np.float64), ref.astype(np.float64))]
    assert min(cos) >= 1.0 - max(2.0 * (1.0 - noise_cos), 2e-4), (min(cos), noise_cos)
    tokens = np.array(dev_tokens)
    bad = np.nonzero(clear & (tokens != ref.argmax(-1)))[0]
    assert bad.size == 0, f"clear steps {bad.tolist()} differ (floor {floor})"
    print(f"clear steps {int(clear.sum())} of {len(tokens)}, noise floor {floor:.3g}, cosine "
          f"{min(cos):.7f} (noise run {noise_cos:.7f})")
    return int(clear.sum()), floor


@pytest.mark.parametrize("fmt,head_fmt", [("int8-row", "int8-row"), ("int4-g32", "int8-row"),
                                          ("int4", "int8-row"), ("int8", "int8")])
def test_tiny_decode_tokens_match_oracle(fmt, head_fmt):
    """Greedy decode of the tiny Qwen3 shape (the reference's test model geometry) through the
    quantized linear layer, the prompt prefilled in one pass: every clear step's token is the
    oracle's (the same model on the CPU with the reference's quantized arithmetic)."""
    from oracle.model import Qwen3Oracle
    from opentpu_b200.model import Qwen3Decoder
    shape = WL.TINY
    W = WL.decoder_weights(shape, seed=1)
    prompt = WL.prompt_ids(shape, 24, seed=2)
    dec = Qwen3Decoder(shape, W, fmt=fmt, head_fmt=head_fmt, max_pos=64)
    tokens, dev = dec.generate(prompt, 12)
    ora = Qwen3Oracle(shape, W, fmt=fmt, head_fmt=head_fmt, rope=lambda p: WL.rope_tables(shape, p))
    clear, _ = _token_parity(tokens, dev, ora, prompt)
    assert clear >= 6


def test_prefill_equals_token_by_token():
    """The prefill's rows through one launch a projection give the same logits as the prompt fed
    token by token (QACT per row: each row's bytes are those of the row alone; the fp32 torch
    attention may differ in its last bits)."""
    from opentpu_b200.model import Qwen3Decoder
    shape = WL.TINY
    W = WL.decoder_weights(shape, seed=4)
    prompt = WL.prompt_ids(shape, 16, seed=5)
    dec = Qwen3Decoder(shape, W, max_pos=32)
    a = dec.prefill(prompt).cpu().numpy()
    dec.reset()
    for tk in prompt:
        b = dec.step(tk)
    b = b.cpu().numpy()
    assert np.abs(a - b).max() <= 1e-4 * np.abs(b).max()


def _qwen3_full_length(fmt, head_fmt):
    """BASELINE configurations 2 and 3 at full length: the seeded Qwen3-0.6B shape, a random
    512-token prompt (prefilled), 64 greedy tokens on the device; the oracle teacher forced on
    the device's tokens over the same 576 positions."""
    from oracle.model import Qwen3Oracle
    from opentpu_b200.model import Qwen3Decoder
    shape = WL.QWEN3_0_6B
    W = WL.decoder_weights(shape, seed=0)
    prompt = WL.prompt_ids(shape, 512, seed=0)
    dec = Qwen3Decoder(shape, W, fmt=fmt, head_fmt=head_fmt, max_pos=576)
    tokens, dev = dec.generate(prompt, 64)
    del dec
    torch.cuda.empty_cache()
    ora = Qwen3Oracle(shape, W, fmt=fmt, head_fmt=head_fmt,
                      rope=lambda p: WL.rope_tables(shape, p))
    return _token_parity(tokens, dev, ora, prompt)


@pytest.mark.slow
def test_qwen3_0_6b_int8_row_decode_512_64_tokens_match_oracle():
    """Configuration 2: int8 per-row layers and head."""
    clear, _ = _qwen3_full_length("int8-row", "int8-row")
    assert clear >= 16


@pytest.mark.slow
def test_qwen3_0_6b_4bit_decode_512_64_tokens_match_oracle():
    """Configuration 3: int4 group-32 fp16-scale layers (weight-only), int8 per-row head."""
    clear, _ = _qwen3_full_length("int4-g32", "int8-row")
    assert clear >= 16
