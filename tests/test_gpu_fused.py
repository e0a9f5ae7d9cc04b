"""The whole decode step as one launch (model.FusedDecoder: the QKV / O / GateUp / Down
projections, the norms, residual adds, attention over the KV cache, SwiGLU, the head and the
greedy token in one persistent kernel; steps feed their tokens to the next on the device)
against the CPU oracle of the same model, under the reference's near-tie rule: on the tiny
Qwen3 shape, and at BASELINE configurations 2 and 3's full length (512-token prompt through the
batched prefill, then 64 fused greedy steps). The down projection's input is one QACT range on
both sides."""
import numpy as np
import pytest

from opentpu_b200 import workloads as WL
from test_gpu_parity import _token_parity

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _run(shape, fmt, head_fmt, prompt_len, n_new, seed_w, seed_p, max_pos):
    from oracle.model import Qwen3Oracle
    from opentpu_b200.model import FusedDecoder, Qwen3Decoder
    W = WL.decoder_weights(shape, seed=seed_w)
    prompt = WL.prompt_ids(shape, prompt_len, seed=seed_p)
    dec = Qwen3Decoder(shape, W, fmt=fmt, head_fmt=head_fmt, max_pos=max_pos, down_chunk=None)
    fused = FusedDecoder(dec)
    tokens, dev = fused.generate(prompt, n_new)
    import ctypes
    from opentpu_b200 import _lib as L
    v = ctypes.c_int(0)
    L.call("otq_status_word", ctypes.addressof(v), 1)
    assert v.value == 0, "a bounded wait ran out"
    assert int(fused.pos[0]) == prompt_len + n_new - 1
    del fused, dec
    torch.cuda.empty_cache()
    ora = Qwen3Oracle(shape, W, fmt=fmt, head_fmt=head_fmt, rope=lambda p: WL.rope_tables(shape, p),
                      down_chunk=None)
    return _token_parity(tokens, dev, ora, prompt)


@pytest.mark.parametrize("fmt", ["int8-row", "int4-g32"])
def test_fused_tiny_decoder_tokens_match_oracle(fmt):
    clear, _ = _run(WL.TINY, fmt, "int8-row", 40, 24, 1, 2, 128)
    assert clear >= 12


def test_fused_step_graph_replays_continue():
    """The step captured once and replayed: every replay decodes the next position from the
    token the previous one chose, as eager launches do."""
    from opentpu_b200.model import FusedDecoder, Qwen3Decoder
    shape = WL.TINY
    W = WL.decoder_weights(shape, seed=3)
    prompt = WL.prompt_ids(shape, 10, seed=4)
    a = FusedDecoder(Qwen3Decoder(shape, W, max_pos=64, down_chunk=None))
    b = FusedDecoder(Qwen3Decoder(shape, W, max_pos=64, down_chunk=None))
    ta, _ = a.generate(prompt, 6, keep_logits=False)
    logits = b.dec.prefill(prompt)
    b.start(int(torch.argmax(logits).item()), len(prompt))
    b.capture()
    tb = [int(b.token[0])]
    for _ in range(5):
        b.graph.replay()
        torch.cuda.synchronize()
        tb.append(int(b.token[0]))
    assert ta == tb
    assert torch.equal(a.logits(), b.logits())


@pytest.mark.parametrize("fmt", ["int8-row", "int4-g32"])
def test_swiglu_epilogue_equals_prologue(fmt):
    """SwiGLU written by the GateUp projection's epilogue (gate / up rows interleaved) and SwiGLU
    read by the Down projection's prologue give the same steps bit for bit."""
    from opentpu_b200.model import FusedDecoder, Qwen3Decoder
    shape = WL.TINY
    W = WL.decoder_weights(shape, seed=5)
    prompt = WL.prompt_ids(shape, 20, seed=6)
    a = FusedDecoder(Qwen3Decoder(shape, W, fmt=fmt, max_pos=64, down_chunk=None))
    b = FusedDecoder(Qwen3Decoder(shape, W, fmt=fmt, max_pos=64, down_chunk=None),
                     swiglu_epilogue=False)
    ta, la = a.generate(prompt, 8)
    tb, lb = b.generate(prompt, 8)
    assert ta == tb
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


@pytest.mark.slow
def test_fused_qwen3_0_6b_int8_row_512_64():
    """Configuration 2 through the fused step."""
    clear, _ = _run(WL.QWEN3_0_6B, "int8-row", "int8-row", 512, 64, 0, 0, 576)
    assert clear >= 16


@pytest.mark.slow
def test_fused_qwen3_0_6b_4bit_512_64():
    """Configuration 3 through the fused step."""
    clear, _ = _run(WL.QWEN3_0_6B, "int4-g32", "int8-row", 512, 64, 0, 0, 576)
    assert clear >= 16
