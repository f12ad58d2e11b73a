"""The tcgen05 tensor-core projection path against the oracle and a float64 product.

Engines with 16 or more slots run every step and prefill projection on the
tensor-core GEMM (TMA-fed, accumulator in tensor memory, split-K with an
ordered reduction); every engine runs the cross K/V projection of a loaded
window on it.  Covered here:

* the cross K/V of a window for every layer (one persistent launch), read
  back from the engine, against ``bf16(bf16(memory) @ bf16(W)^T + bf16(b))``
  computed in float64, for ragged frame counts, float32 and bfloat16 memory,
  from 2 layers at d128 to 12 layers at d1024;
* a 16-slot teacher-forced decode (ragged prefixes and frame counts) against
  the oracle's bf16 mode, with the same logit and near-tie rules as the
  CUDA-core path;
* the properties the CUDA-core path has, on tensor cores: a prefilled prefix
  gives bit-identical results to forcing it token by token, and a slot's
  tokens do not depend on the other slots.
"""

import ctypes as C
import dataclasses

import numpy as np
import pytest
import torch

import scenarios as sc
from helpers import (LOGIT_WITHIN_FRACTION, TOKEN_AGREEMENT, cuda_engine, logit_error, logit_within, loader, masked,
                     near_tie, oracle_engine, prefill_compare, weights)
from sheetsage2_refined_b200 import _lib
from sheetsage2_refined_b200.grammar import TableGrammar
from sheetsage2_refined_b200.vocab_table import OUT, SOS
from sheetsage2_refined_b200.weights import memory_array

pytestmark = pytest.mark.gpu
BATCH = 16  # the smallest engine whose step projections run on tensor cores


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def bf16(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).float().numpy()


def cross_kv(eng, name: str) -> np.ndarray:
    """A cross K or V buffer of the engine ("cross_k" = layer 0, "cross_k.<l>" = layer l),
    [batch, heads, frames, 64] as float32."""

    ptr, numel, dtype = C.c_void_p(), C.c_int64(), C.c_int32()
    _lib.check(eng._lib.s2r_get_buffer(eng._ctx, name.encode(), C.byref(ptr), C.byref(numel), C.byref(dtype)))
    assert dtype.value == 1
    raw = torch.as_tensor(_DeviceView(ptr.value, numel.value), device=eng.device)
    torch.cuda.synchronize()
    cfg = eng.config
    return raw.view(torch.bfloat16).float().cpu().numpy().reshape(eng.batch, cfg.heads, eng.frames, 64)


class _DeviceView:
    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False), "version": 3,
                                         "strides": None}


def expected_cross(config, seed, memory: np.ndarray, which: str, layer: int = 0) -> np.ndarray:
    """[heads, frames, 64]: bf16(bf16(memory) @ bf16(W)^T + bf16(b)) with a float64 sum."""

    st = weights(config, seed)
    w = bf16(st[f"layers.{layer}.cross_attn.{which}.weight"]).astype(np.float64)
    b = bf16(st[f"layers.{layer}.cross_attn.{which}.bias"]).astype(np.float64)
    x = bf16(memory).astype(np.float64)
    y = bf16((x @ w.T + b).astype(np.float32))
    scale = np.abs(x) @ np.abs(w).T + np.abs(b)  # sum of |terms|: bounds the float32 accumulation error
    split = lambda a: a.reshape(memory.shape[0], config.heads, 64).transpose(1, 0, 2)  # noqa: E731
    return split(y), split(scale)


def assert_bf16_close(got: np.ndarray, want, what: str):
    """Equal except where the float32 sum moves a value across a bf16 rounding boundary.

    ``want`` = (float64 result rounded to bf16, sum of |terms|).  A value may differ by one bf16
    ulp, plus the float32 accumulation error, which the sum of |terms| bounds (2^-20 of it: far
    above what K <= 1024 float32 additions of these magnitudes produce, far below a wrong term);
    that only matters where the terms cancel to a value much smaller than themselves.
    """

    want, scale = want
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -126))) - 7)
    diff = np.abs(got - want)
    exact = float((diff == 0).mean())
    print(f"{what}: {exact:.4%} bit-equal, max {float((diff / ulp).max()):.2f} ulp, "
          f"max {float((diff / scale).max()):.2e} of the sum of |terms|")
    assert (diff <= ulp * 1.0001 + scale * 2.0 ** -20).all(), what
    assert exact >= 0.98, what


@pytest.mark.parametrize("config,frames_engine,frames,batch", [
    (sc.C1, sc.C1_FRAMES, sc.C1_FRAMES, 2),   # two full frame tiles, 4 feature tiles (2 layers x 2D = 512)
    (sc.C1, sc.C1_FRAMES, 200, 2),            # ragged last frame tile
    (sc.REAL_TINY, sc.REAL_FRAMES, 37, 2),    # one partial frame tile; a feature tile holds a layer's K and V
    (sc.C1, sc.C1_FRAMES, 131, BATCH),        # batched engine
], ids=["c1-full", "c1-ragged", "tiny", "c1-batch16"])
def test_cross_kv_projection(config, frames_engine, frames, batch):
    """Every layer's cross K/V (one launch for all layers) against a float64 product."""

    seed = sc.C1_SEED if config is sc.C1 else sc.REAL_SEED
    grammar = sc.c1_grammar() if config is sc.C1 else TableGrammar(config.vocab_size)
    eng = cuda_engine(config, seed, grammar, batch, frames_engine)
    mem = memory_array(frames_engine, config.width, 77)[0]
    slot = batch - 1
    eng.load(slot, mem, [SOS, OUT], None, frames, target=64)
    got = {}
    for layer in range(config.layers):
        for which in "kv":
            got[layer, which] = cross_kv(eng, f"cross_{which}.{layer}")[slot, :, :frames]
            assert_bf16_close(got[layer, which], expected_cross(config, seed, mem[:frames], which, layer),
                              f"layer {layer} cross {which.upper()}")
    assert np.array_equal(cross_kv(eng, "cross_k")[slot], cross_kv(eng, "cross_k.0")[slot])
    # bfloat16 memory takes the GEMM without the conversion kernel: same values bit for bit
    eng.load(0, torch.from_numpy(mem).to(torch.bfloat16), [SOS, OUT], None, frames, target=64)
    for (layer, which), want in got.items():
        assert np.array_equal(cross_kv(eng, f"cross_{which}.{layer}")[0, :, :frames], want)


def test_cross_kv_projection_d1024_every_layer():
    """The single-song decoder's shape: 12 layers of [Wck; Wcv] [2048, 1024] over 1,500 frames in one
    persistent launch (1,152 tiles of 128 frames x 256 features over the SMs)."""

    cfg = dataclasses.replace(sc.C2, max_tokens=128)
    frames = sc.C2_FRAMES
    grammar = TableGrammar(cfg.vocab_size)
    eng = cuda_engine(cfg, sc.C2_SEED, grammar, 1, frames)
    mem = memory_array(frames, cfg.width, 78)[0]
    eng.load(0, torch.from_numpy(mem).to(torch.bfloat16), [SOS, OUT], None, frames - 3, target=8)
    for layer in (0, 5, cfg.layers - 1):
        for which in "kv":
            got = cross_kv(eng, f"cross_{which}.{layer}")[0, :, :frames - 3]
            assert_bf16_close(got, expected_cross(cfg, sc.C2_SEED, mem[:frames - 3], which, layer),
                              f"layer {layer} cross {which.upper()}")


def load_ragged(engines, rng, vocab):
    """Load every slot with its own memory, prefix length (2..6) and frame count."""

    plans = []
    for slot in range(BATCH):
        prefix = [SOS, OUT] + rng.integers(4, vocab, slot % 5).tolist()
        frames = sc.C1_FRAMES - 11 * slot
        plans.append((slot, 300 + slot, prefix, frames))
    for eng in engines:
        load = loader(eng, sc.C1.width, sc.C1_FRAMES)
        for slot, seed, prefix, frames in plans:
            load(slot, seed, prefix, None, frames, 10_000)


def test_batched_step_vs_oracle_bf16():
    grammar = sc.c1_grammar()
    eng = cuda_engine(sc.C1, sc.C1_SEED, grammar, BATCH, sc.C1_FRAMES)
    assert eng.step_launches == 11 * sc.C1.layers + 2  # a LayerNorm launch per LayerNorm'd projection
    ora = oracle_engine(sc.C1, sc.C1_SEED, grammar, BATCH, sc.C1_FRAMES)
    rng = np.random.default_rng(5)
    load_ragged([eng, ora], rng, sc.C1.vocab_size)
    max_err, within, count, same, steps, ties = 0.0, 0, 0, 0, 0, 0
    for k in range(24):
        forced = rng.integers(4, sc.C1.vocab_size, BATCH).astype(np.int64)
        allowed = ora.grammar.allowed(ora.state)
        lg_e, gr_e = eng.step_debug(forced)
        lg_o, gr_o = ora.step(forced=forced)
        for slot in range(BATCH):
            max_err = max(max_err, logit_error(lg_e[slot], lg_o[slot]))
            w, n = logit_within(lg_e[slot], lg_o[slot])
            within, count = within + w, count + n
            steps += 1
            if gr_e[slot] == gr_o[slot]:
                same += 1
            else:
                ml = masked(lg_o[slot], allowed[slot], ora.logit_bias)
                assert near_tie(ml, int(gr_e[slot]), int(gr_o[slot])), (k, slot, gr_e[slot], gr_o[slot])
                ties += 1
    print(f"batch {BATCH} on tensor cores vs oracle bf16: logit error {max_err:.3f}, "
          f"{within / count:.5f} within 2e-2, greedy {same}/{steps} ({ties} near-ties)")
    assert max_err <= 1.0
    assert within / count >= LOGIT_WITHIN_FRACTION
    assert same / steps >= TOKEN_AGREEMENT


@pytest.mark.parametrize("n,exact", [(9, True), (152, False), (300, False)], ids=["8-rows", "150-rows", "298-rows"])
def test_batched_prefill_equals_token_by_token(n, exact):
    """A prefilled prefix against forcing it token by token on a 16-slot engine.  Chunks of up to 8
    rows run the decode step's attention (one cluster per row and head): bit-identical.  Longer chunks
    (128 rows and the rest) run the tensor-core prefill attention, whose online softmax adds in
    another order: the same logits within the parity tolerance."""

    rng = np.random.default_rng(11)
    grammar = sc.c1_grammar()
    seq = [SOS, OUT] + rng.integers(4, sc.C1.vocab_size, 320).tolist()
    a = cuda_engine(sc.C1, sc.C1_SEED, grammar, BATCH, sc.C1_FRAMES)
    b = cuda_engine(sc.C1, sc.C1_SEED, grammar, BATCH, sc.C1_FRAMES)
    slot = 5
    loader(a, sc.C1.width, sc.C1_FRAMES)(slot, 3, seq[:n], None, 200, 10_000)
    loader(b, sc.C1.width, sc.C1_FRAMES)(slot, 3, seq[:2], None, 200, 10_000)
    forced = np.full(BATCH, -1, np.int64)
    for k in range(n - 2):
        forced[slot] = seq[2 + k]
        b.step_debug(forced, want_logits=False)
    for k in range(8):
        forced[slot] = seq[n + k]
        la, ga = a.step_debug(forced)
        lb, gb = b.step_debug(forced)
        prefill_compare(la[slot], lb[slot], ga[slot], gb[slot], exact, k)


def test_batched_slot_independence_bit_exact():
    alone = cuda_engine(sc.C1, sc.C1_SEED, sc.c1_grammar(), BATCH, sc.C1_FRAMES)
    busy = cuda_engine(sc.C1, sc.C1_SEED, sc.c1_grammar(), BATCH, sc.C1_FRAMES)
    la = loader(alone, sc.C1.width, sc.C1_FRAMES)
    lb = loader(busy, sc.C1.width, sc.C1_FRAMES)
    la(9, 21, [SOS, OUT, 77], None, 180, 96)
    for slot in range(BATCH):
        if slot != 9:
            lb(slot, 40 + slot, [SOS, OUT], None, 256 - slot, 20 + 7 * slot)
    busy.run(5)
    lb(9, 21, [SOS, OUT, 77], None, 180, 96)
    alone.run(96)
    busy.run(96)
    assert alone.take(9) == busy.take(9)


def test_no_tensor_core_flag_keeps_cuda_core_projections():
    eng = cuda_engine(sc.C1, sc.C1_SEED, sc.c1_grammar(), BATCH, sc.C1_FRAMES, flags=_lib.S2R_FLAG_NO_TENSOR_CORE)
    assert eng.step_launches == 6 * sc.C1.layers + 1  # CUDA-core projections, fused attention
