"""Host-side logic that needs no GPU: the C library loads and exports every
declared symbol, conv planning (geometry, workspace, packed-weight rows),
sampler schedules and coefficients vs the oracle, and weight packing."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    names = []
    for header in (ROOT / "include").glob("*.h"):
        names += re.findall(r"^LDB_API [^(]*?\b(ldb_\w+)\s*\(", header.read_text(), flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from lesiondiffusion_mlx_b200 import _lib

    lib = _lib.library()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.ldb_version() == 4


def test_errors_are_reported_without_a_device():
    from lesiondiffusion_mlx_b200 import _lib

    desc = _lib.ConvDesc(batch=1, depth=2, height=2, width=2, in_channels=16, x_ld=20, out_channels=8, out_ld=8,
                         res_ld=8, mode=0, exact=0, out_dtype=0, act=0, output_scale=1.0)
    size = ctypes.c_size_t(0)
    with pytest.raises(_lib.LdbError, match="multiple of 8"):
        _lib.call("ldb_conv3d_workspace_size", ctypes.byref(desc), ctypes.byref(size))
    desc.x_ld = 16
    desc.mode = 9
    with pytest.raises(_lib.LdbError, match="unknown conv mode"):
        _lib.call("ldb_conv3d_workspace_size", ctypes.byref(desc), ctypes.byref(size))


def test_conv_descriptor_of_another_layout_is_rejected():
    """A binding that mirrors an older or shorter ``ldb_conv_desc`` (no
    ``struct_size`` first field, or a struct that stops before ``clock``) gets
    LDB_ERR_INVALID from every descriptor entry point instead of a launch that
    reads past the struct it passed."""
    from lesiondiffusion_mlx_b200 import _lib

    good = _lib.ConvDesc(batch=1, depth=2, height=2, width=2, in_channels=16, x_ld=16, out_channels=8, out_ld=8,
                         res_ld=8, mode=0, exact=0, out_dtype=0, act=0, output_scale=1.0)
    size = ctypes.c_size_t(0)
    _lib.call("ldb_conv3d_workspace_size", ctypes.byref(good), ctypes.byref(size))
    assert good.struct_size == ctypes.sizeof(_lib.ConvDesc) == 80

    class ShortDesc(ctypes.Structure):
        # the version-1 layout: no struct_size, and it ends at depth_halo
        _fields_ = [(n, ctypes.c_int) for n in ("batch", "depth", "height", "width", "in_channels", "x_ld",
                                                "out_channels", "out_ld", "res_ld", "mode", "exact", "out_dtype",
                                                "act")] + [("output_scale", ctypes.c_float), ("depth_halo", ctypes.c_int)]

    # a padded buffer keeps the library's read of the full struct inside our own memory
    buf = (ctypes.c_char * ctypes.sizeof(_lib.ConvDesc))()
    short = ShortDesc.from_buffer(buf)
    short.batch, short.depth, short.height, short.width = 1, 2, 2, 2
    short.in_channels, short.x_ld, short.out_channels, short.out_ld, short.res_ld = 16, 16, 8, 8, 8
    short.output_scale = 1.0
    lib = _lib.library()
    rows, k = ctypes.c_int(0), ctypes.c_int(0)
    stats_host = (ctypes.c_double * 2)()  # non-null, so the descriptor check is what fails
    stats_ptr = ctypes.cast(stats_host, ctypes.c_void_p)
    for name, args in (("ldb_conv3d_workspace_size", (ctypes.byref(size),)),
                       ("ldb_conv3d_weight_rows", (ctypes.byref(rows), ctypes.byref(k))),
                       ("ldb_conv3d_fwd", (None, None, None, None, None, None, None, 0)),
                       ("ldb_conv3d_fwd_gn_stats", (None, None, None, None, None, None, stats_ptr, None, 0))):
        fn = getattr(lib, name)
        if name.startswith("ldb_conv3d_fwd"):
            rc = fn(None, ctypes.cast(buf, ctypes.POINTER(_lib.ConvDesc)), *args)
        else:
            rc = fn(ctypes.cast(buf, ctypes.POINTER(_lib.ConvDesc)), *args)
        assert rc == -1, name  # LDB_ERR_INVALID
        assert b"struct_size" in lib.ldb_last_error(), name
    good.struct_size = 72  # the version-2 layout (no max_ctas)
    with pytest.raises(_lib.LdbError, match="struct_size 72"):
        _lib.call("ldb_conv3d_workspace_size", ctypes.byref(good), ctypes.byref(size))
    good.struct_size = ctypes.sizeof(_lib.ConvDesc)
    good.max_ctas = -1
    with pytest.raises(_lib.LdbError, match="max_ctas"):
        _lib.call("ldb_conv3d_workspace_size", ctypes.byref(good), ctypes.byref(size))


@pytest.mark.parametrize("cin,cout,exact,rows,k", [(128, 128, False, 128, 27 * 128), (8, 8, False, 16, 27 * 16),
                                                    (512, 384, False, 512, 27 * 512), (4, 16, True, 16, 2 * 27 * 16),
                                                    (256, 40, False, 64, 27 * 256)])
def test_conv_weight_geometry(cin, cout, exact, rows, k):
    from lesiondiffusion_mlx_b200 import _lib

    desc = _lib.ConvDesc(batch=1, depth=1, height=1, width=1, in_channels=cin,
                         x_ld=max(8, 2 * ((cin + 15) // 16) * 16 if exact else (cin + 7) // 8 * 8),
                         out_channels=cout, out_ld=cout, res_ld=cout, mode=0, exact=int(exact), out_dtype=0, act=0,
                         output_scale=1.0)
    r, kt = ctypes.c_int(0), ctypes.c_int(0)
    _lib.call("ldb_conv3d_weight_rows", ctypes.byref(desc), ctypes.byref(r), ctypes.byref(kt))
    assert (r.value, kt.value) == (rows, k)


def test_split_k_workspace_only_for_small_grids():
    from lesiondiffusion_mlx_b200 import _lib

    def ws(d, h, w, cin):
        desc = _lib.ConvDesc(batch=1, depth=d, height=h, width=w, in_channels=cin, x_ld=cin, out_channels=512,
                             out_ld=512, res_ld=512, mode=0, exact=0, out_dtype=0, act=0, output_scale=1.0)
        size = ctypes.c_size_t(0)
        _lib.call("ldb_conv3d_workspace_size", ctypes.byref(desc), ctypes.byref(size))
        return size.value

    assert ws(8, 10, 10, 512) > 0  # 800 voxels: too few tiles, K is split
    assert ws(32, 40, 40, 128) == 0  # 400 brick tiles fill the GPU


def test_conv_geometry_uses_input_extents():
    from lesiondiffusion_mlx_b200.conv import MODE_CONV, MODE_STRIDE2, MODE_UP2, PackedWeight, conv_geometry

    x = torch.empty((2, 5, 7, 9, 24))[..., :20]
    conv = PackedWeight(torch.empty(0), "conv", 20, 40, False)
    assert conv_geometry(tuple(x.shape), tuple(x.stride()), conv) == (MODE_CONV, (5, 7, 9), 24, 20)
    assert conv_geometry(tuple(x.shape), tuple(x.stride()), conv, stride=2) == (MODE_STRIDE2, (3, 4, 5), 24, 20)
    up = PackedWeight(torch.empty(0), "up", 20, 40, False)
    assert conv_geometry(tuple(x.shape), tuple(x.stride()), up) == (MODE_UP2, (10, 14, 18), 24, 20)
    with pytest.raises(ValueError, match="dense over voxels"):
        y = torch.empty((2, 5, 7, 10, 24))[:, :, :, :9, :20]
        conv_geometry(tuple(y.shape), tuple(y.stride()), conv)


def test_upsample_fold_matches_conv_of_upsampled_input():
    """The packed parity fold reproduces conv(upsample2(x)) (checked on CPU in float64)."""
    from lesiondiffusion_mlx_b200.conv import pack_upsample_weight
    from oracle import ops as oops

    rng = np.random.default_rng(4)
    w = torch.from_numpy(rng.normal(size=(8, 16, 3, 3, 3)).astype(np.float32))
    x = torch.from_numpy(rng.normal(size=(1, 16, 3, 4, 5)))
    ref = torch.nn.functional.conv3d(oops.upsample_nearest2(x), w.double(), padding=1)
    got = oops.upsample_conv(x, w, None, dtype=torch.float64, compute=torch.float64)
    assert torch.allclose(got, ref, atol=1e-5)
    packed = pack_upsample_weight(w)
    assert packed.exact and packed.kind == "up" and packed.tensor.shape == (8 * 16, 2 * 8 * 16)


def test_sampler_tables_match_oracle():
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, Dpmpp2mSampler
    from oracle import samplers as osamp

    with np.load(ROOT / "tests/golden/reference_fixtures.npz") as g:
        acp = g["dpmpp_2m/linet_25.alphas_cumprod"]
    d = DdimSampler(acp, 200)
    ref = osamp.ddim_coefficients(acp, 200)
    assert d.timesteps == tuple(ref["timesteps"])
    np.testing.assert_array_equal(d.sigmas, ref["sigmas"])
    np.testing.assert_array_equal(d.coefficients[0, :4], [ref["alphas"][-1], ref["previous"][-1],
                                                           ref["sigmas"][-1], ref["sqrt_one_minus"][-1]])
    p = Dpmpp2mSampler(acp, 50)
    ts, coeffs = osamp.dpm_coefficients(acp, 50)
    assert p.timesteps == ts
    np.testing.assert_array_equal(p.coefficients, coeffs)
    with pytest.raises(ValueError):
        DdimSampler(acp, 3)


def test_one_step_ddim_table_has_positive_strides():
    """A one-step DDIM schedule's coefficient table (reversed into execution
    order) is a real copy: torch cannot wrap a view with a negative stride."""
    import torch

    from lesiondiffusion_mlx_b200.sampling import DdimSampler

    alphas = np.linspace(0.9999, 0.02, 1000).astype(np.float32)
    for steps in (1, 2, 50):
        table = DdimSampler(alphas, steps).coefficients
        assert table.shape == (steps, 5) and all(s > 0 for s in table.strides)
        assert torch.from_numpy(table).shape == (steps, 5)


def test_entry_points_reject_rows_their_strides_do_not_cover():
    """Row strides shorter than the rows they step over, and element types a
    kernel does not read, fail with an error before any launch (checked
    without a device: the pointers are host placeholders never dereferenced)."""
    from lesiondiffusion_mlx_b200 import _lib

    buf = (ctypes.c_char * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p).value
    cases = [
        ("ldb_layer_norm_ex", (None, p, _lib.LDB_F16, 32, p, p, 1e-5, p, 64, 4, 64, 0), "x_ld 32 < 64"),
        ("ldb_dense_small", (None, p, 8, p, None, p, 64, 2, 64, 16, 0, 0, _lib.LDB_F16, 0), "must cover K 16"),
        ("ldb_dense_small", (None, p, 16, p, None, p, 64, 2, 64, 16, 0, 0, _lib.LDB_BF16, 0), "out dtype"),
        ("ldb_hu_map", (None, p, _lib.LDB_F16, 0, 10, p), "x_ld must be positive"),
        ("ldb_hu_map", (None, p, _lib.LDB_BF16, 1, 10, p), "input dtype"),
        ("ldb_resize_nearest", (None, p, 1, 2, 2, 2, 16, 8, p, 4, 4, 4, 16), "cover the 16-byte rows"),
        ("ldb_timestep_embedding", (None, p, None, 1, 2, 32, p, _lib.LDB_BF16), "out dtype"),
    ]
    for name, args, message in cases:
        with pytest.raises(_lib.LdbError, match=message):
            _lib.call(name, *args)


def test_ctypes_signatures_match_the_header():
    """Every ctypes signature of the binding has the parameters of its
    declaration in ``include/ldb200.h``, in order and by kind (pointer, int,
    float, double, 64-bit integer), and the declared return type: a binding
    that drifts from the header (a parameter added on one side only) fails here
    instead of shifting every later argument at run time."""
    from lesiondiffusion_mlx_b200 import _lib

    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "ldb200.h").read_text(), flags=re.S)

    def c_kind(param: str) -> str:
        param = re.sub(r"\bconst\b", "", param).strip()
        if "*" in param or param.startswith("ldb_stream_t"):
            return "ptr"
        base = re.sub(r"\s+\w+$", "", param).strip()  # drop the parameter name
        return {"long long": "i64", "unsigned int": "uint", "unsigned long long": "u64", "size_t": "u64"}.get(base, base)

    def py_kind(t) -> str:
        if t is ctypes.c_void_p or t is ctypes.c_char_p or (isinstance(t, type) and issubclass(t, ctypes._Pointer)):
            return "ptr"
        # (ctypes makes c_size_t the same type as c_ulonglong on 64-bit Linux: both are "u64")
        return {ctypes.c_int: "int", ctypes.c_float: "float", ctypes.c_double: "double", ctypes.c_size_t: "u64",
                ctypes.c_longlong: "i64", ctypes.c_uint: "uint", ctypes.c_ulonglong: "u64"}[t]

    declared = re.findall(r"LDB_API\s+([^;(]*?)\b(ldb_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S)
    assert len(declared) == len(declared_symbols())
    for ret, name, params in declared:
        params = params.strip()
        kinds = [] if params in ("", "void") else [c_kind(p) for p in params.split(",")]
        assert [py_kind(t) for t in _lib.SIGNATURES[name]] == kinds, name
        assert py_kind(_lib._RESTYPES.get(name, ctypes.c_int)) == c_kind(ret.strip() + " r"), name


def test_conv_descriptor_fields_match_the_header():
    """``_lib.ConvDesc`` lists the fields of ``ldb_conv_desc`` in the header's
    order with the same kinds (the size check alone would pass two swapped
    fields of one type)."""
    from lesiondiffusion_mlx_b200 import _lib

    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "ldb200.h").read_text(), flags=re.S)
    body = re.search(r"typedef struct \{(.*?)\}\s*ldb_conv_desc;", text, flags=re.S).group(1)
    fields = []
    for decl in filter(None, (d.strip() for d in body.split(";"))):
        kind = "ptr" if "*" in decl else decl.split()[0]
        names = decl.replace("*", " ").split(None, 1)[1] if kind != "ptr" else decl.split("*")[-1]
        fields += [(n.strip(), kind) for n in names.split(",")]
    kinds = {ctypes.c_int: "int", ctypes.c_float: "float", ctypes.c_void_p: "ptr"}
    assert [(n, kinds[t]) for n, t in _lib.ConvDesc._fields_] == fields
