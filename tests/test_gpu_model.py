"""The whole encoder through the public C API (nextera_load / nextera_encode*) on a
B200, against the CPU oracle on the same GGUF files and inputs.

Bar (north star): last_hidden_state within 1e-3 relative error (L2 norm of the
difference over the L2 norm of the oracle's) and token cosine >= 0.9999; pooled
embeddings likewise.  Within a batch, a sequence's result must not depend on
the rest of the batch: bit-identical (nexterabert.h).
"""
import ctypes

import numpy as np
import pytest

import cases
import synth_model as sm

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
COS_MIN = 0.9999


@pytest.fixture(scope="module")
def lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpulib import load_lib
    return load_lib()


class Model:
    def __init__(self, L, path):
        self.L = L
        p = L.nextera_default_params()
        self.h = L.nextera_load(str(path).encode(), p)
        assert self.h, f"nextera_load failed for {path}"
        self.C = L.nextera_n_embd(self.h)

    def encode(self, tokens, lengths, types=None, normalize=True, hidden=True):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lengths = np.ascontiguousarray(lengths, np.int32)
        T = int(lengths.sum())
        hid = np.empty((T, self.C), np.float32) if hidden else None
        pooled = np.empty((len(lengths), self.C), np.float32)
        i32 = ctypes.POINTER(ctypes.c_int32)
        f32 = ctypes.POINTER(ctypes.c_float)
        ty = None if types is None else np.ascontiguousarray(types, np.int32)
        rc = self.L.nextera_encode_segments(self.h, tokens.ctypes.data_as(i32),
                                            None if ty is None else ty.ctypes.data_as(i32),
                                            lengths.ctypes.data_as(i32), len(lengths),
                                            None if hid is None else hid.ctypes.data_as(f32),
                                            pooled.ctypes.data_as(f32), int(normalize))
        return rc, hid, pooled

    def close(self):
        self.L.nextera_free(self.h)


def compare(got, want, what):
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    cos = np.sum(got * want, 1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
    print(f"{what}: rel err {rel:.3e}, min token cosine {cos.min():.8f}, bit-identical {np.mean(got == want):.6f}")
    assert rel <= REL_TOL, f"{what}: relative error {rel:.3e}"
    assert cos.min() >= COS_MIN, f"{what}: min token cosine {cos.min():.6f}"
    return rel, float(cos.min())


@pytest.mark.parametrize("preset,seed", [("Q4_K_M", 0), ("Q8_0", 1), ("Q5_K_M", 2), ("Q4_0", 3)])
def test_tiny_model_matches_oracle(lib, oracle, preset, seed):
    path = sm.cached_model("tiny", sm.tiny_hparams(), preset, seed=seed)
    m = Model(lib, path)
    tok, lens = cases.model_batch(1000, seed=7)
    rc, hid, pooled = m.encode(tok, lens)
    assert rc == 0
    o = oracle.load(path)
    want_h, want_p = o.encode(tok, lens)
    compare(hid, want_h, "hidden")
    compare(pooled, want_p, "pooled")
    rc, _, raw = m.encode(tok, lens, normalize=False, hidden=False)
    _, want_raw = o.encode(tok, lens, normalize=False, hidden=False)
    compare(raw, want_raw, "pooled (not normalised)")
    m.close()
    o.close()


def test_batch_invariance_bit_exact(lib):
    """A sequence encodes to the same bits alone and inside a mixed batch."""
    path = sm.cached_model("tiny", sm.tiny_hparams(), "Q4_K_M", seed=0)
    m = Model(lib, path)
    tok, lens = cases.model_batch(1000, seed=7)
    _, hid, pooled = m.encode(tok, lens)
    start = np.concatenate([[0], np.cumsum(lens)[:-1]])
    for d in range(len(lens)):
        s0, n = int(start[d]), int(lens[d])
        _, h1, p1 = m.encode(tok[s0:s0 + n], lens[d:d + 1])
        assert np.array_equal(h1, hid[s0:s0 + n]), d
        assert np.array_equal(p1[0], pooled[d]), d
    m.close()


def test_segments_ssmax_and_ntk(lib, oracle):
    hp = sm.tiny_hparams(n_types=2, ssmax_mode="ssmax", ntk_train_len=64)
    path = sm.cached_model("tiny_seg", hp, "Q5_K_M", seed=4)
    m = Model(lib, path)
    o = oracle.load(path)
    tok = sm.random_tokens(200, hp.n_vocab, seed=1)
    L = np.array([200], np.int32)            # beyond ntk_train_len: stretched RoPE base
    types = (np.arange(200) >= 100).astype(np.int32)
    rc, hid, pooled = m.encode(tok, L, types=types)
    assert rc == 0
    wh, wp = o.encode(tok, L, types=types)
    compare(hid, wh, "hidden")
    compare(pooled, wp, "pooled")
    # beyond ntk_train_length, sequences must be encoded one at a time (error 1)
    rc, _, _ = m.encode(np.concatenate([tok, tok]), np.array([200, 200], np.int32))
    assert rc == 1
    m.close()
    o.close()


def test_debug_layers(lib, oracle):
    path = sm.cached_model("tiny", sm.tiny_hparams(), "Q8_0", seed=1)
    m = Model(lib, path)
    o = oracle.load(path)
    tok, lens = cases.model_batch(1000, seed=9)
    for n in (1, 2, 3):
        lib.nextera_debug_set_layers(m.h, n)
        _, hid, _ = m.encode(tok, lens)
        want, _ = o.encode(tok, lens, n_layers=n)
        compare(hid, want, f"{n} layers")
    m.close()
    o.close()


def test_bad_inputs_return_codes(lib):
    path = sm.cached_model("tiny", sm.tiny_hparams(), "Q8_0", seed=1)
    m = Model(lib, path)
    rc, _, _ = m.encode(np.array([1, 2, 3], np.int32), np.array([3, 0], np.int32))
    assert rc == 1                                       # empty sequence
    rc, _, _ = m.encode(np.array([1, 2, 5000], np.int32), np.array([3], np.int32))
    assert rc == 1                                       # token id out of range
    rc, _, _ = m.encode(np.array([1, 2, 3], np.int32), np.array([3], np.int32), types=np.array([0, 1, 0], np.int32))
    assert rc == 0                                       # types are ignored by a file without segments
    m.close()


def test_encode_device_matches_host(lib):
    import torch
    from gpulib import P, dev, host
    path = sm.cached_model("tiny", sm.tiny_hparams(), "Q4_K_M", seed=0)
    m = Model(lib, path)
    tok, lens = cases.model_batch(1000, seed=7)
    _, hid, pooled = m.encode(tok, lens)
    dt = dev(tok)
    dh = torch.empty(hid.shape, dtype=torch.float32, device="cuda")
    dp = torch.empty(pooled.shape, dtype=torch.float32, device="cuda")
    i32 = ctypes.POINTER(ctypes.c_int32)
    lens = np.ascontiguousarray(lens, np.int32)
    rc = lib.nextera_encode_device(m.h, P(dt), None, lens.ctypes.data_as(i32), len(lens), P(dh), P(dp), 1,
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    assert np.array_equal(host(dh), hid)
    assert np.array_equal(host(dp), pooled)
    m.close()


def test_cfg3_full_model_q4km(lib, oracle):
    """Config 3: the full 18-layer model in Q4_K_M, one sequence of 512 ids."""
    path = sm.cached_model("full", sm.full_hparams(), "Q4_K_M", seed=0)
    m = Model(lib, path)
    assert b"linear layers: 141 int8" in lib.nextera_system_info(m.h)
    tok = sm.random_tokens(512, 50368, seed=0)
    L = np.array([512], np.int32)
    rc, hid, pooled = m.encode(tok, L)
    assert rc == 0
    o = oracle.load(path)
    wh, wp = o.encode(tok, L)
    rel, cos = compare(hid, wh, "hidden")
    compare(pooled, wp, "pooled")
    print(f"cfg3: hidden rel err {rel:.2e}, min token cosine {cos:.8f}")
    m.close()
    o.close()


def test_repeated_shapes_replay_graphs_bit_exact(lib, oracle):
    """A batch shape seen before runs as a recorded CUDA graph: new token ids, the same bits as the
    eager forward, whatever ran in between (other shapes, hidden on / off, segments)."""
    hp = sm.tiny_hparams(n_types=2)
    path = sm.cached_model("tiny_seg", hp, "Q4_K_M", seed=3)
    m = Model(lib, path)
    fresh = Model(lib, path)                    # a second context that never repeats a shape
    shapes = [np.array([5, 17, 40], np.int32), np.array([64, 1, 130], np.int32)]
    for it in range(4):
        for si, lens in enumerate(shapes):
            rng = np.random.default_rng(100 * it + si)
            tok = rng.integers(0, 1000, int(lens.sum())).astype(np.int32)
            types = rng.integers(0, 2, int(lens.sum())).astype(np.int32) if si == 1 else None
            want_hidden = it != 2
            rc, hid, pooled = m.encode(tok, lens, types=types, hidden=want_hidden)
            assert rc == 0
            # the reference result of this call: a context seeing the shape for the first time
            fresh.close()
            fresh = Model(lib, path)
            rc2, hid2, pooled2 = fresh.encode(tok, lens, types=types, hidden=True)
            assert rc2 == 0
            assert np.array_equal(pooled, pooled2), (it, si)
            if want_hidden:
                assert np.array_equal(hid, hid2), (it, si)
    # graphs were used: later calls of a shape launch the recorded kernels (same launch count)
    n0 = lib.nextera_debug_launches(m.h)
    rc, _, _ = m.encode(np.zeros(int(shapes[0].sum()), np.int32), shapes[0])
    assert rc == 0 and lib.nextera_debug_launches(m.h) > n0
    m.close()
    fresh.close()


@pytest.mark.parametrize("preset", ["F16", "F32"])
def test_float_encoder_files_are_refused_at_load(lib, capfd, preset):
    # The reference runs float matrices on ggml's mul_mat (src/nexterabert.cpp:1140-1142); this
    # build has only the int8 path for encoder linears, so such a file is refused at load: NULL and
    # a message naming the tensor, as for any other file it cannot run.
    path = sm.cached_model("tiny", sm.tiny_hparams(), preset, seed=0)
    h = lib.nextera_load(str(path).encode(), lib.nextera_default_params())
    err = capfd.readouterr().err
    assert not h
    assert "is not a quantized matrix this build can expand to int8" in err
    assert "'blocks." in err


@pytest.mark.parametrize("preset", ["Q4_K_M", "Q8_0"])
def test_full_model_edge_lengths_match_reference(lib, reflib, preset):
    """The full model on a batch of edge-case lengths against the reference compiled here:
    1-token documents, lengths around the 8-key groups of the score lanes, around the band
    half-width (128) and window (256), and around 2048, where the reference's attention switches to
    blocked keys (src/nexterabert.cpp:776-780, :810-837)."""
    path = sm.cached_model("full", sm.full_hparams(), preset, seed=0)
    lens = np.array([1, 2, 7, 8, 9, 127, 129, 255, 256, 257, 2047, 2048, 2049], np.int32)
    tok = sm.random_tokens(int(lens.sum()), 50368, seed=31)
    m = Model(lib, path)
    rc, hid, pooled = m.encode(tok, lens)
    assert rc == 0
    r = reflib.load(path, 0)
    try:
        wh, wp = reflib.encode(r, tok, lens)
    finally:
        reflib.L.nextera_free(r)
    compare(hid, wh, f"hidden ({preset})")
    compare(pooled, wp, f"pooled ({preset})")
    print(f"{preset}: hidden bit-identical fraction {np.mean(hid == wh):.6f}")
    m.close()
