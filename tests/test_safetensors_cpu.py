"""The checkpoint reader without a GPU: tensors, dtypes,
shapes, bytes and __metadata__ read back exactly; F16 / BF16 widened exactly;
every malformed header refused whole."""
import json
import struct

import numpy as np
import pytest

import st_file


def _open(path):
    import ltx25_b200 as L
    return L.SafeTensors(path)


def test_reads_back_every_tensor(tmp_path):
    rng = np.random.default_rng(1)
    t = {
        "model.diffusion_model.transformer_blocks.0.attn1.to_q.weight":
            rng.integers(0, 2 ** 32, (8, 16), dtype=np.uint64).astype(np.uint32),
        "model.diffusion_model.transformer_blocks.0.attn1.to_q.scales":
            rng.standard_normal((8, 1)).astype(np.float16),
        "a.f32": rng.standard_normal((3, 5, 2)).astype(np.float32),
        "b.bf16": rng.integers(0, 2 ** 16, (7,), dtype=np.uint16),
        "scalar": np.float32(2.5).reshape(()),
        "empty": np.zeros((0, 4), np.float32),
    }
    p = st_file.write(tmp_path / "m.safetensors", t, metadata={"lora_alpha": "450", "x": "yé"},
                      bf16=("b.bf16",))
    st = _open(p)
    assert sorted(st.names()) == sorted(t)
    for name, a in t.items():
        dt, shape, _, nbytes = st.info(st.find(name))
        assert shape == list(np.shape(a)), name
        assert nbytes == np.asarray(a).nbytes, name
        assert np.array_equal(st.raw(name), np.frombuffer(np.asarray(a).tobytes(order="C"),
                                                          np.uint8)), name
    assert st.info(st.find("b.bf16"))[0] == "BF16"
    assert st.find("nope") == -1
    assert st.metadata("lora_alpha") == "450"
    assert st.metadata("x") == "yé"
    assert st.metadata("missing") is None


def test_widens_half_and_bfloat_exactly(tmp_path):
    # every finite f16 bit pattern, the infinities and a NaN
    h = np.arange(0, 2 ** 16, dtype=np.uint32).astype(np.uint16)
    halfs = h.view(np.float16)
    bf = np.array([0x0000, 0x8000, 0x3F80, 0xBF80, 0x7F80, 0xFF80, 0x0001, 0x7F7F, 0x4049],
                  np.uint16)
    p = st_file.write(tmp_path / "f.safetensors", {"h": halfs, "b": bf}, bf16=("b",))
    st = _open(p)
    got = st.read_f32("h")
    want = halfs.astype(np.float32)
    fin = np.isfinite(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])
    gb = st.read_f32("b")
    assert np.array_equal(gb.view(np.uint32), bf.astype(np.uint32) << 16)


def _raw(tmp_path, header_obj=None, header_bytes=None, data=b"", length=None):
    h = header_bytes if header_bytes is not None else json.dumps(header_obj).encode()
    p = tmp_path / "bad.safetensors"
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(h) if length is None else length))
        f.write(h)
        f.write(data)
    return p


@pytest.mark.parametrize("case", [
    "short", "length_past_end", "not_object", "bad_json", "unknown_dtype", "offsets_vs_shape",
    "past_data", "duplicate", "trailing", "float_shape", "missing_offsets", "negative_dim",
    "repeated_shape", "repeated_dtype", "nine_dims"])
def test_refuses_malformed_headers(tmp_path, case):
    import ltx25_b200 as L
    ok = {"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    data = b"\0" * 8
    if case == "short":
        p = tmp_path / "s.safetensors"
        p.write_bytes(b"\x01\x02")
    elif case == "length_past_end":
        p = _raw(tmp_path, ok, data=data, length=10 ** 6)
    elif case == "not_object":
        p = _raw(tmp_path, header_bytes=b"[1, 2]", data=data)
    elif case == "bad_json":
        p = _raw(tmp_path, header_bytes=b'{"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]', data=data)
    elif case == "unknown_dtype":
        p = _raw(tmp_path, {"t": {"dtype": "F8_E4M3", "shape": [2], "data_offsets": [0, 2]}}, data=data)
    elif case == "offsets_vs_shape":
        p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, data=data)
    elif case == "past_data":
        p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, data=data)
    elif case == "duplicate":
        p = _raw(tmp_path, header_bytes=b'{"t": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}, '
                 b'"t": {"dtype": "F32", "shape": [1], "data_offsets": [4, 8]}}', data=data)
    elif case == "trailing":
        p = _raw(tmp_path, header_bytes=json.dumps(ok).encode() + b" x", data=data)
    elif case == "float_shape":
        p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [2.0], "data_offsets": [0, 8]}}, data=data)
    elif case == "missing_offsets":
        p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [2]}}, data=data)
    elif case == "repeated_shape":
        # [1] then [2]: appended, the shape would read [1, 2] and match the data
        p = _raw(tmp_path, header_bytes=b'{"t": {"dtype": "F32", "shape": [1], "shape": [2], '
                 b'"data_offsets": [0, 8]}}', data=data)
    elif case == "repeated_dtype":
        p = _raw(tmp_path, header_bytes=b'{"t": {"dtype": "F16", "dtype": "F32", "shape": [2], '
                 b'"data_offsets": [0, 8]}}', data=data)
    elif case == "nine_dims":
        # consistent with its data, but more dimensions than the ABI's shape holds
        p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [1] * 8 + [2],
                                  "data_offsets": [0, 8]}}, data=data)
    else:
        p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [-2], "data_offsets": [0, 8]}}, data=data)
    with pytest.raises(L.LtxError) as e:
        _open(p)
    assert e.value.code == -2, str(e.value)
    print(case, e.value)


def test_missing_file_and_nulls():
    import ltx25_b200 as L
    with pytest.raises(L.LtxError) as e:
        _open("/nonexistent/dir/x.safetensors")
    assert e.value.code == -7
    lib = L.load()
    assert lib.ltx_st_count(None) == 0
    assert lib.ltx_st_name(None, 0) is None
    assert lib.ltx_st_find(None, b"x") == -1
    assert lib.ltx_st_metadata(None, b"x") is None
    assert lib.ltx_block_load_st(None, None, b"") == -1
    assert lib.ltx_lora_load_st(None, None, b"", 1, 1, 1.0, None) == -1
    lib.ltx_st_close(None)


def test_random_headers_never_crash(tmp_path):
    """Property: any header bytes either parse into tensors that lie inside
    the data, or are refused with LTX_E_SHAPE -- never a crash or a tensor
    reaching past the file."""
    from hypothesis import given, settings, strategies as s
    import ltx25_b200 as L

    ident = s.text(alphabet="abc._", min_size=1, max_size=6)
    entry = s.fixed_dictionaries({
        "dtype": s.sampled_from(["F32", "F16", "BF16", "U32", "I8", "X9", ""]),
        "shape": s.lists(s.integers(-2, 6), max_size=3),
        "data_offsets": s.lists(s.integers(-4, 80), min_size=0, max_size=3),
    })
    header = s.dictionaries(ident, entry, max_size=4)
    path = tmp_path / "fuzz.safetensors"

    @settings(max_examples=300, deadline=None)
    @given(header, s.integers(0, 96), s.booleans())
    def run(h, data_len, garble):
        raw = json.dumps(h).encode()
        if garble and raw:
            raw = raw[: len(raw) // 2]
        with open(path, "wb") as f:
            f.write(struct.pack("<Q", len(raw)))
            f.write(raw)
            f.write(b"\x5a" * data_len)
        try:
            st = L.SafeTensors(path)
        except L.LtxError as e:
            assert e.code == -2, str(e)
            return
        for i in range(len(st)):
            _, shape, ptr, nbytes = st.info(i)
            assert nbytes <= data_len
        st.close()

    run()


def test_device_free_apis_refuse_nulls():
    """The adapter, connector and adaLN entry points refuse null handles
    without touching a device."""
    import ltx25_b200 as L
    lib = L.load()
    assert lib.ltx_connector_create(None, 4, 64, 1, 8, 1, 10000.0, 4096, 1, None) == -1
    assert lib.ltx_connector_load_st(None, None, b"") == -1
    assert lib.ltx_connector_finalize(None) == -1
    assert lib.ltx_connector_reserve(None, 8) == -1
    assert lib.ltx_connector_forward(None, None, None, 8, 8, None) == -1
    assert lib.ltx_connector_last_error(None) == b"null connector"
    lib.ltx_connector_destroy(None)
    assert lib.ltx_adaln_run(None, 1.0, None, None, 0) == -1
    assert lib.ltx_adaln_create(None, None, None, None, None, None, 8, 8, None) == -1
    assert lib.ltx_adaln_load_st(None, b"", None, None, 0) == -1
    lib.ltx_adaln_free(None)
    assert lib.ltx_patchify(None, None, None, None, None, 0, None, 0, None, 1, 128, 64, None) == -1
    assert lib.ltx_output_head(None, None, None, None, None, None, None, 0, 1, 64, 8, None) == -1


def test_eight_dimensions_is_the_limit(tmp_path):
    """A tensor of 8 dimensions (the ABI's shape slots) opens and reports
    all of them; the nine-dimension case above is refused."""
    import ltx25_b200 as L
    p = _raw(tmp_path, {"t": {"dtype": "F32", "shape": [1] * 7 + [2],
                              "data_offsets": [0, 8]}}, data=b"\0" * 8)
    st = _open(p)
    _, shape, _, nbytes = st.info(0)
    assert list(shape) == [1] * 7 + [2] and nbytes == 8
    st.close()
