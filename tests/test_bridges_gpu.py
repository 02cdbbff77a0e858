"""Stored 4-bit data and GEMM operands on the GPU.

* ``brc_pack_nibbles_hi`` / ``brc_unpack_nibbles_hi`` equal the reference's
  ``pack_nibbles`` / ``unpack_nibbles`` (``_formats.py:227-260``): against the
  golden bytes the reference wrote and the oracle on ragged sizes.
* ``attach_gemm_operands`` rebuilds exactly the side operands the cast wrote
  (scale atoms, tensor-core packed codes, INT4 tiles), byte for byte.
* save (packed or not) -> load onto the GPU gives the same tensors, the same
  GEMM operands, and the same GEMM results bit for bit.
"""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "bridge_ref.safetensors")


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _raw():
    from safetensors import safe_open
    with safe_open(GOLDEN, framework="pt") as f:
        return f.metadata(), {k: f.get_tensor(k) for k in f.keys()}


def _call(name, *args):
    from breccia_b200 import _lib
    _lib.call(name, *args, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("name", ["nvfp4", "int4_sym", "int4_asym", "int4_u_g64"])
def test_pack_unpack_golden(name):
    _, raw = _raw()
    codes = raw[f"{name}.data"].cuda().contiguous()
    n = codes.numel()
    packed = torch.empty(n // 2, dtype=torch.uint8, device="cuda")
    _call("brc_pack_nibbles_hi", codes.data_ptr(), n, packed.data_ptr())
    assert torch.equal(packed.cpu(), raw[f"{name}.packed_ref"])
    back = torch.empty_like(codes)
    lo = torch.empty(n // 2, dtype=torch.uint8, device="cuda")
    _call("brc_unpack_nibbles_hi", packed.data_ptr(), n, back.data_ptr(), lo.data_ptr())
    assert torch.equal(back, codes)
    c = codes.cpu().numpy().ravel()
    np.testing.assert_array_equal(lo.cpu().numpy(), (c[0::2] & 15) | ((c[1::2] & 15) << 4))


@pytest.mark.parametrize("n", [2, 14, 16, 18, 1000, 4096 + 6, (1 << 20) + 10])
def test_pack_unpack_ragged_vs_oracle(n):
    from oracle import codec
    g = torch.Generator().manual_seed(n)
    # high nibbles set too: the kernels must use the low nibble only, as pack_nibbles does
    codes = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8)
    cd = codes.cuda()
    packed = torch.empty(n // 2, dtype=torch.uint8, device="cuda")
    _call("brc_pack_nibbles_hi", cd.data_ptr(), n, packed.data_ptr())
    want = codec.pack_nibbles(codes.numpy())
    np.testing.assert_array_equal(packed.cpu().numpy(), want)
    back = torch.empty(n, dtype=torch.uint8, device="cuda")
    _call("brc_unpack_nibbles_hi", packed.data_ptr(), n, back.data_ptr(), None)
    np.testing.assert_array_equal(back.cpu().numpy(), codec.unpack_nibbles(want, n))
    lo = torch.empty(n // 2, dtype=torch.uint8, device="cuda")
    _call("brc_pack_codes_lo", cd.data_ptr(), n, lo.data_ptr())
    c = codes.numpy()
    np.testing.assert_array_equal(lo.cpu().numpy(), (c[0::2] & 15) | ((c[1::2] & 15) << 4))


def test_entry_point_errors():
    from breccia_b200 import _lib
    st = torch.cuda.current_stream().cuda_stream
    buf = torch.empty(64, dtype=torch.uint8, device="cuda")
    assert _lib.lib().brc_pack_nibbles_hi(buf.data_ptr(), 3, buf.data_ptr(), st) == _lib.BRC_ERR_SHAPE
    assert _lib.lib().brc_pack_nibbles_hi(None, 4, buf.data_ptr(), st) == _lib.BRC_ERR_NULL
    assert _lib.lib().brc_unpack_nibbles_hi(buf.data_ptr(), 4, None, None, st) == _lib.BRC_ERR_NULL
    assert _lib.lib().brc_pack_nibbles_hi(buf.data_ptr() + 1, 4, buf.data_ptr(), st) == \
        _lib.BRC_ERR_ALIGN
    assert _lib.lib().brc_int4_tiles(buf.data_ptr(), 8, 128, buf.data_ptr(), None, 0,
                                     buf.data_ptr(), buf.data_ptr(), None, st) == \
        _lib.BRC_ERR_UNSUPPORTED
    assert _lib.lib().brc_scale_atoms(buf.data_ptr(), 0, 4, buf.data_ptr(), st) == _lib.BRC_OK


def _recipes():
    from breccia_b200.types import MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling
    return {
        "mxfp8": MXFP8BlockScaling(),
        "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
        "nvfp4": NVFP4BlockScaling(),
        "int4_sym": INT4Scaling(group_size=128),
        "int4_sym_u_f32": INT4Scaling(group_size=128, signed=False, scale_dtype="fp32"),
        "int4_asym": INT4Scaling(group_size=128, signed=False, symmetric=False),
        "int4_asym_f32": INT4Scaling(group_size=128, signed=False, symmetric=False,
                                     scale_dtype="fp32"),
    }


def _shapes(rname):
    if rname.startswith("int4"):
        return [(16, 128), (48, 384), (3, 32, 256), (4096, 1024)]
    return [(1, 64), (130, 96), (257, 1056), (2, 70, 512), (4096, 1024)]


def _strip(st):
    """The same ScaledTensor with fresh data storage (so no side operands)."""
    return type(st)(data=st.data.clone(), scale=st.scale.clone(), recipe=st.recipe,
                    layout=st.layout,
                    zero_point=None if st.zero_point is None else st.zero_point.clone())


@pytest.mark.parametrize("rname", list(_recipes()))
def test_attach_equals_cast_side(rname):
    import breccia_b200 as bb
    r = _recipes()[rname]
    for shape in _shapes(rname):
        g = torch.Generator(device="cuda").manual_seed(sum(shape))
        x = torch.randn(shape, generator=g, device="cuda") * 3
        st = bb.cast(x, r)
        want = bb.gemm_operands(st)
        bare = _strip(st)
        assert bb.gemm_operands(bare) == {}
        bb.attach_gemm_operands(bare)
        got = bb.gemm_operands(bare)
        keys = {k for k, v in want.items() if v is not None}
        assert keys <= {k for k, v in got.items() if v is not None}, (shape, keys, got.keys())
        for k in keys:
            assert torch.equal(got[k].view(torch.uint8), want[k].view(torch.uint8)), (shape, k)


@pytest.mark.parametrize("pack", [False, True])
@pytest.mark.parametrize("rname", ["mxfp8", "nvfp4", "int4_sym", "int4_asym"])
def test_save_load_round_trip_gemm(tmp_path, rname, pack):
    import breccia_b200 as bb
    from breccia_b200 import bridges
    r = _recipes()[rname]
    g = torch.Generator(device="cuda").manual_seed(7)
    N, K = 512, 1024
    w = bb.cast(torch.randn(N, K, generator=g, device="cuda") * 0.05, r)
    path = str(tmp_path / "w.safetensors")
    bridges.save_safetensors({"w": w}, path, pack_4bit=pack)
    from safetensors import safe_open
    with safe_open(path, framework="pt") as f:
        keys = set(f.keys())
    packed = pack and rname in ("nvfp4", "int4_sym", "int4_asym")
    assert ("w.data_packed" in keys) == packed and ("w.data" in keys) == (not packed)
    lw = bridges.load_safetensors(path, device="cuda")["w"]
    assert lw.data.is_cuda and torch.equal(lw.data, w.data) and torch.equal(lw.scale, w.scale)
    if w.zero_point is not None:
        assert torch.equal(lw.zero_point, w.zero_point)
    want, got = bb.gemm_operands(w), bb.gemm_operands(lw)
    for k, v in want.items():
        if v is not None:
            assert torch.equal(got[k].view(torch.uint8), v.view(torch.uint8)), k
    # the same tensor-core kernels run on the loaded weight: identical results
    if rname.startswith("int4"):
        a = torch.randn(4, K, generator=g, device="cuda").to(torch.bfloat16)
        out0 = bb.linear(a, w, out_dtype=torch.float32)
        out1 = bb.linear(a, lw, out_dtype=torch.float32)
    else:
        a = bb.cast(torch.randn(256, K, generator=g, device="cuda"), r)
        out0 = bb.linear(a, w, out_dtype=torch.float32)
        out1 = bb.linear(a, lw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    if rname.startswith("int4"):
        # the INT4 kernel adds row-block partial sums with shared-memory atomics, so
        # the float32 summation order (and the last bits) varies between runs
        assert ((out0 - out1).abs().max() / out0.abs().max()).item() <= 1e-6
    else:
        assert torch.equal(out0, out1)


def test_load_reference_file_onto_gpu():
    """The reference-written file loads onto the GPU with GEMM operands
    attached; its dequantized values equal the CPU-loaded tensors' (oracle)."""
    import breccia_b200 as bb
    from breccia_b200 import bridges
    from oracle import cast as ocast
    cpu = bridges.load_safetensors(GOLDEN)
    gpu = bridges.load_safetensors(GOLDEN, device="cuda")
    for name, st in gpu.items():
        c = cpu[name]
        assert torch.equal(st.data.cpu().view(torch.uint8), c.data.view(torch.uint8))
        lay = c.layout
        ltup = (lay.name, lay.block_m, lay.block_n) if lay.name == "per_block_mn" else \
            (lay.name, getattr(lay, "block_size", None))
        q = ocast.Q(data=c.data.view(torch.uint8).numpy(), scale=c.scale.numpy(), layout=ltup,
                    recipe=c.recipe,
                    zero_point=None if c.zero_point is None else c.zero_point.numpy())
        deq = bb.dequantize(st).cpu().numpy()
        ref = ocast.dequantize(q)
        gn, rn = np.isnan(deq), np.isnan(ref)
        np.testing.assert_array_equal(gn, rn)
        np.testing.assert_array_equal(deq[~gn].view(np.uint32), ref[~rn].view(np.uint32))
    assert "sf_mma" in bb.gemm_operands(gpu["nvfp4"]) and "packed" in bb.gemm_operands(gpu["nvfp4"])
    assert "sf_mma" in bb.gemm_operands(gpu["mxfp8"])
    assert "int4_tiles" in bb.gemm_operands(gpu["int4_asym"])
    assert "int4_tiles" in bb.gemm_operands(gpu["int4_sym"])


def test_dlpack_zero_copy_of_outputs():
    """The reference's DLPack bridge (src/breccia/bridges/_dlpack.py:18-67)
    hands this backend's CUDA outputs on without copying: torch's DLPack
    export carries the float8 dtypes, and consumers without float8 take the
    uint8 view of the same bytes."""
    import breccia_b200 as bb
    x = torch.randn(64, 256, device="cuda")
    for r in (bb.Float8CurrentScaling(), bb.MXFP8BlockScaling(), bb.NVFP4BlockScaling()):
        st = bb.cast(x, r)
        for t in (st.data, st.scale):
            back = torch.from_dlpack(t.__dlpack__())
            assert back.data_ptr() == t.data_ptr() and back.dtype == t.dtype
        u8 = torch.from_dlpack(st.data.view(torch.uint8))
        assert u8.data_ptr() == st.data.data_ptr()


# ------------------------------------------------------------ TransformerEngine
# TE is not installed in this image; a module with TE's Float8Tensor
# constructor and DType enum (the attribute shape the reference's own
# validation uses, benchmarks/modal_te_validate.py:130-174) stands in for it.

@pytest.fixture
def fake_te(monkeypatch):
    import enum
    import sys
    import types as pytypes

    class DType(enum.Enum):
        kFloat8E4M3 = 7
        kFloat8E5M2 = 8

    class Float8Tensor:
        def __init__(self, *, data, fp8_scale_inv, fp8_dtype):
            self._data, self._scale_inv, self._fp8_dtype = data, fp8_scale_inv, fp8_dtype

        def dequantize(self):
            fdt = torch.float8_e4m3fn if self._fp8_dtype == DType.kFloat8E4M3 else torch.float8_e5m2
            return self._data.view(fdt).to(torch.float32) * self._scale_inv

    te = pytypes.ModuleType("transformer_engine")
    te_pt = pytypes.ModuleType("transformer_engine.pytorch")
    te_pt.Float8Tensor = Float8Tensor
    te_torch = pytypes.ModuleType("transformer_engine_torch")
    te_torch.DType = DType
    te.pytorch = te_pt
    for name, mod in (("transformer_engine", te), ("transformer_engine.pytorch", te_pt),
                      ("transformer_engine_torch", te_torch)):
        monkeypatch.setitem(sys.modules, name, mod)
    return Float8Tensor, DType


@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_transformer_engine_round_trip_shares_buffers(fake_te, fmt):
    """GPU per-tensor output -> Float8Tensor -> ScaledTensor: the same device
    buffers throughout, TE's dequantize equals this backend's bit for bit."""
    import breccia_b200 as bb
    from breccia_b200 import bridges
    Float8Tensor, DType = fake_te
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(256, 512, generator=g) * 3).cuda()
    st = bb.cast(x, bb.Float8CurrentScaling(fp8_format=fmt))
    te_t = bridges.to_transformer_engine(st)
    assert isinstance(te_t, Float8Tensor)
    assert te_t._fp8_dtype == (DType.kFloat8E4M3 if fmt == "E4M3" else DType.kFloat8E5M2)
    assert te_t._data.dtype == torch.uint8 and tuple(te_t._scale_inv.shape) == (1,)
    assert te_t._data.data_ptr() == st.data.data_ptr()
    assert te_t._scale_inv.data_ptr() == st.scale.data_ptr()
    assert torch.equal(te_t.dequantize().view(torch.int32), bb.dequantize(st).view(torch.int32))
    back = bridges.from_transformer_engine(te_t)
    assert back.recipe.name == "delayed" and back.recipe.fp8_format == fmt
    assert back.scale.ndim == 0 and back.data.data_ptr() == st.data.data_ptr()
    assert torch.equal(bb.dequantize(back), bb.dequantize(st))
    with pytest.raises(NotImplementedError):
        bridges.to_transformer_engine(bb.cast(x, bb.MXFP8BlockScaling()))


def test_transformer_engine_missing_raises():
    from breccia_b200 import bridges
    import breccia_b200 as bb
    st = bb.cast(torch.randn(16, 32).cuda(), bb.Float8CurrentScaling())
    with pytest.raises(ImportError, match="TransformerEngine is required"):
        bridges.to_transformer_engine(st)
