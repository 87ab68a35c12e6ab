"""C-ABI library: it loads, exports every symbol declared in include/*.h, and its
host-side argument validation answers before any device work (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

from fast_infer_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(fi_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.fi_version() >= 100


def _declarations():
    """name -> parameter list (C text) of every function declared in include/*.h."""
    out = {}
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for name, params in re.findall(r"\b(fi_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
            params = " ".join(params.split())
            out[name] = [] if params in ("", "void") else [x.strip() for x in params.split(",")]
    return out


def test_ctypes_signatures_match_the_header():
    """Every binding in _lib.SIGNATURES has the header's argument count and, per
    argument, a matching kind (pointer / int64 / int / size_t / float), and the
    FI_* constants the Python layer mirrors equal the header's."""
    decls = _declarations()
    assert set(decls) == set(_lib.SIGNATURES)
    scalar = {"int64_t": ctypes.c_int64, "int": ctypes.c_int, "size_t": ctypes.c_size_t,
              "float": ctypes.c_float, "double": ctypes.c_double}
    for name, params in decls.items():
        argtypes = _lib.SIGNATURES[name][1]
        assert len(argtypes) == len(params), (name, len(argtypes), len(params))
        for i, (c, py) in enumerate(zip(params, argtypes)):
            if "*" in c:
                assert py in (ctypes.c_void_p, ctypes.c_char_p) or \
                    issubclass(py, ctypes._Pointer), (name, i, c, py)
            else:
                ctype = c.replace("const ", "").rsplit(" ", 1)[0].strip()
                assert scalar[ctype] is py, (name, i, c, py)
    text = "".join(h.read_text() for h in (ROOT / "include").glob("*.h"))
    defines = dict(re.findall(r"#define\s+(FI_[A-Z0-9_]+)\s+(-?\d+)\b", text))
    mirrored = [n for n in dir(_lib) if re.fullmatch(r"FI_[A-Z0-9_]+", n) and n in defines]
    assert {"FI_OK", "FI_ERR_WORKSPACE", "FI_DEVERR_TIMEOUT", "FI_STATIC_WEIGHTS"} <= set(mirrored)
    for n in mirrored:
        assert getattr(_lib, n) == int(defines[n]), n


def _nul():
    return ctypes.c_void_p(0)


def test_prefill_rejects_bad_head_dim_and_groups():
    lib = _lib.load()
    s4 = _lib.strides(1, 1, 1, 1)
    st = lib.fi_prefill_fwd(1, 1, 1, 1, 1, 24, 8, 16, 64, s4, s4, s4, s4, 0.1, None, None)
    assert st == _lib.FI_ERR_UNSUPPORTED
    assert b"head_dim" in lib.fi_last_error()
    st = lib.fi_prefill_fwd(1, 1, 1, 1, 1, 24, 7, 16, 128, s4, s4, s4, s4, 0.1, None, None)
    assert st == _lib.FI_ERR_INVALID_ARG
    st = lib.fi_prefill_fwd(None, None, None, None, 1, 24, 8, 16, 128, s4, s4, s4, s4, 0.1,
                            None, None)
    assert st == _lib.FI_ERR_INVALID_ARG
    # empty problems are a no-op
    assert lib.fi_prefill_fwd(None, None, None, None, 0, 24, 8, 16, 128, s4, s4, s4, s4, 0.1,
                              None, None) == _lib.FI_OK


def test_decode_validation_and_workspace_size():
    lib = _lib.load()
    s3, s4, s2 = _lib.strides(1, 1, 1), _lib.strides(1, 1, 1, 1), _lib.strides(1, 1)
    args = lambda **kw: dict(dict(num_tokens=10, max_ctx=0, batch=2, hq=24, hkv=8, d=128,
                                  nb=4, bs=64, mb=4), **kw)

    def call(a, ptr=1):
        return lib.fi_paged_decode(ptr, ptr, ptr, ptr, ptr, None, a["num_tokens"], a["max_ctx"],
                                   a["batch"], a["hq"], a["hkv"], a["d"], a["nb"], a["bs"],
                                   a["mb"], s3, s4, s4, s3, s2, 0.1, 0, None, 0, None, None)
    assert call(args(d=64)) == _lib.FI_ERR_UNSUPPORTED
    assert call(args(bs=16)) == _lib.FI_ERR_UNSUPPORTED
    assert call(args(hq=25)) == _lib.FI_ERR_INVALID_ARG
    assert call(args(hq=72, hkv=8)) == _lib.FI_ERR_UNSUPPORTED  # group of 9
    assert call(args(num_tokens=4 * 64 + 1)) == _lib.FI_ERR_INVALID_ARG
    assert call(args(), ptr=None) == _lib.FI_ERR_INVALID_ARG
    # workspace: none for a single split, proportional to splits otherwise
    assert lib.fi_paged_decode_workspace_size(2, 24, 8, 128, 64, 64, 0) == 0
    ws = lib.fi_paged_decode_workspace_size(2, 24, 8, 128, 4096, 64, 8)
    assert ws == 2 * 24 * (64 // 8) * (128 * 4 + 8)
    # too-small workspace is reported before launch
    st = lib.fi_paged_decode(1, 1, 1, 1, 1, None, 4096, 0, 2, 24, 8, 128, 64, 64, 64,
                             s3, s4, s4, s3, s2, 0.1, 8, None, 0, None, None)
    assert st == _lib.FI_ERR_WORKSPACE


def test_automatic_split_rule():
    """The automatic split-KV choice, read back through the workspace it needs. Grids
    that would leave most SMs idle (at least two SMs per sequence x KV head) split each
    over a thread-block cluster of 2, 4 or 8 CTAs (4 to 32 pages per CTA) that merge
    in shared memory: no workspace. Otherwise about
    SMs / (2 x sequences x KV heads) splits per sequence, 4 to 32 pages each, and 32
    pages per split once that is one split (148 SMs: a B200, and the count the library
    assumes with no device)."""
    import torch
    if torch.cuda.is_available() and \
            torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("rule values below are for 148 SMs")
    lib = _lib.load()

    def expect(batch, hq, hkv, max_ctx, sms=148):
        pages = -(-max_ctx // 64)
        cs = min(sms // (batch * hkv), 8, pages // 4)
        cs = 8 if cs >= 8 else 4 if cs >= 4 else 2 if cs >= 2 else 1
        if cs > 1 and -(-pages // cs) <= 32:
            return 0  # cluster merge in shared memory
        splits = sms // (2 * batch * hkv)
        pps = 32 if splits <= 1 else min(32, max(4, -(-pages // splits)))
        n = -(-pages // pps)
        return 0 if n <= 1 else batch * hq * n * (128 * 4 + 8)

    cases = [(64, 24, 8, 4096, 2),     # config 3: 32 pages per split, two splits at most
             (16, 24, 8, 1280, 1),     # the stack's decode step: unsplit
             (16, 6, 2, 1280, 1),      # its 4-GPU share: clusters of 4 CTAs
             (256, 24, 8, 4096, 2),    # config 5
             (256, 3, 1, 4096, 2),     # config 5, one KV head per rank (8-GPU partition)
             (1, 24, 8, 8192, 1),      # one long sequence: clusters of 8, 16 pages each
             (1, 24, 8, 32768, 16),    # too long for a cluster: 16 splits of 32 pages
             (2, 3, 1, 4096, 1),       # one KV head: clusters of 8
             (2, 3, 1, 500, 1)]        # 8 pages: clusters of 2 (4 pages per CTA)
    for batch, hq, hkv, ctx, nsplit in cases:
        ws = lib.fi_paged_decode_workspace_size(batch, hq, hkv, 128, ctx, 64, 0)
        assert ws == expect(batch, hq, hkv, ctx), (batch, hq, hkv, ctx)
        assert ws == (0 if nsplit == 1 else batch * hq * nsplit * (128 * 4 + 8))


def test_kv_write_validation():
    lib = _lib.load()
    s4, s2 = _lib.strides(1, 1, 1, 1), _lib.strides(1, 1)
    st = lib.fi_kv_write(None, None, None, None, None, None, 0, None, 1, 1, 8, 128, 4, 64, 4,
                         s4, s4, s4, s4, s2, None, None)
    assert st == _lib.FI_ERR_INVALID_ARG
    st = lib.fi_kv_write(1, 1, 1, 1, 1, None, 250, None, 1, 10, 8, 128, 4, 64, 4,
                         s4, s4, s4, s4, s2, None, None)
    assert st == _lib.FI_ERR_INVALID_ARG  # positions 250..259 need a 5th block
    assert lib.fi_kv_write(None, None, None, None, None, None, 0, None, 0, 1, 8, 128, 4, 64, 4,
                           s4, s4, s4, s4, s2, None, None) == _lib.FI_OK


def test_python_wrappers_reject_cpu_tensors():
    import torch
    from fast_infer_b200.kernels.attention import flash_attention, paged_attention
    q = torch.zeros(1, 2, 4, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        flash_attention(q, q, q)
    with pytest.raises(ValueError, match="CUDA"):
        paged_attention(q[:, :, 0], torch.zeros(2, 64, 2, 128, dtype=torch.float16),
                        torch.zeros(2, 64, 2, 128, dtype=torch.float16),
                        torch.zeros(1, 2, dtype=torch.int32), 64, 5)
    # reference semantics without touching the device: num_tokens == 0 -> zeros
    out = paged_attention(q[:, :, 0], None, None, None, 64, 0)
    assert out.shape == (1, 2, 128) and not out.any()


def test_int4_validation():
    lib = _lib.load()
    s2 = _lib.strides(16, 1)
    # K not a multiple of groupsize; groupsize not a multiple of 32; M beyond the fused path
    assert lib.fi_int4_gemm(1, 1, 1, 1, 4, 64, 200, 128, s2, s2, s2, s2,
                            None, None) == _lib.FI_ERR_INVALID_ARG
    assert lib.fi_int4_gemm(1, 1, 1, 1, 4, 64, 160, 16, s2, s2, s2, s2,
                            None, None) == _lib.FI_ERR_UNSUPPORTED
    assert lib.fi_int4_gemm(1, 1, 1, 1, 65, 64, 256, 128, s2, s2, s2, s2,
                            None, None) == _lib.FI_ERR_UNSUPPORTED
    assert b"dense GEMM" in lib.fi_last_error()
    # misaligned x row stride / packed row stride, null pointers
    assert lib.fi_int4_gemm(16, 16, 16, 16, 4, 64, 256, 128, _lib.strides(260, 1), s2, s2, s2,
                            None, None) == _lib.FI_ERR_ALIGNMENT
    assert lib.fi_int4_gemm(16, 16, 16, 16, 4, 64, 256, 128, _lib.strides(256, 1),
                            _lib.strides(130, 1), s2, s2, None, None) == _lib.FI_ERR_ALIGNMENT
    assert lib.fi_int4_gemm(None, 16, 16, 16, 4, 64, 256, 128, s2, s2, s2, s2,
                            None, None) == _lib.FI_ERR_INVALID_ARG
    # empty problems are a no-op
    assert lib.fi_int4_gemm(None, None, None, None, 0, 64, 256, 128, s2, s2, s2, s2,
                            None, None) == _lib.FI_OK
    # dequant / quantize argument checks
    assert lib.fi_int4_dequant(1, 1, 1, 8, 200, 128, s2, s2, s2, None) == _lib.FI_ERR_INVALID_ARG
    assert lib.fi_int4_dequant(1, 1, 16, 8, 256, 128, _lib.strides(128, 1), s2,
                               _lib.strides(250, 1), None) == _lib.FI_ERR_ALIGNMENT
    assert lib.fi_int4_quantize(1, 1, 1, 8, 256, 127, s2, s2, s2, None) == _lib.FI_ERR_INVALID_ARG
    assert lib.fi_int4_quantize(1, 1, 1, 0, 256, 128, s2, s2, s2, None) == _lib.FI_OK


def test_small_gemm_validation():
    from fast_infer_b200 import _lib
    lib = _lib.load()
    s2 = _lib.strides(1, 1)
    s3 = _lib.strides(1, 1, 1)
    s4 = _lib.strides(1, 1, 1, 1)
    # more than 16 rows, K not a multiple of 64, null pointers: rejected on the host
    assert lib.fi_small_gemm(None, None, None, None, None, 1e-5, 17, 8, 64, s2, s2, s2, None,
                             0, None, None) == _lib.FI_ERR_UNSUPPORTED
    assert lib.fi_small_gemm(None, None, None, None, None, 1e-5, 4, 8, 100, s2, s2, s2, None,
                             0, None, None) == _lib.FI_ERR_UNSUPPORTED
    assert lib.fi_small_gemm(None, None, None, None, None, 1e-5, 4, 8, 64, s2, s2, s2, None,
                             0, None, None) == _lib.FI_ERR_INVALID_ARG
    assert lib.fi_small_gemm(None, None, None, None, None, 1e-5, 0, 8, 64, s2, s2, s2, None,
                             0, None, None) == _lib.FI_OK
    assert lib.fi_small_gemm_folded(None, None, None, None, 1e-5, 17, 8, 64, s2, s2, s2, None,
                                    0, None, None) == _lib.FI_ERR_UNSUPPORTED
    assert lib.fi_small_gemm_folded(None, None, None, None, 1e-5, 4, 8, 64, s2, s2, s2, None,
                                    _lib.FI_STATIC_WEIGHTS, None, None) == _lib.FI_ERR_INVALID_ARG
    # flags: FI_STATIC_WEIGHTS is the only bit; any other is rejected before anything else
    for flags in (2, 1 << 40, -1):
        assert lib.fi_small_gemm(None, None, None, None, None, 1e-5, 0, 8, 64, s2, s2, s2,
                                 None, flags, None, None) == _lib.FI_ERR_INVALID_ARG
        assert lib.fi_small_gemm_folded(None, None, None, None, 1e-5, 4, 8, 64, s2, s2, s2,
                                        None, flags, None, None) == _lib.FI_ERR_INVALID_ARG
        assert lib.fi_qkv_rope_kv_write(None, None, 1e-5, 4, 64, 3, 1, 128, s2, s2, None, None,
                                        16, 128, None, None, s3, None, None, None, 8, 64, 2,
                                        s4, s4, s2, flags, None, None) == _lib.FI_ERR_INVALID_ARG
    assert "unknown flags" in lib.fi_last_error().decode()


def test_peer_gather_host_checks():
    """Peer gather set-up and call checks that answer before any device work: the
    region size (this rank's output buffers plus an 8-byte landing slot per 4-byte
    word of every buffer, plus a small local state), and the argument checks of
    fi_peer_gather / fi_peer_alloc / fi_peer_open (null handles close and free as
    no-ops)."""
    lib = _lib.load()
    assert lib.fi_peer_gather_bytes(0, 16, 1536) == 0
    assert lib.fi_peer_gather_bytes(3, 0, 1536) == 0
    assert lib.fi_peer_gather_bytes(3, 16, -1) == 0
    for nbuf, rows, row_total in ((3, 16, 2 * 768), (28, 16, 8 * 768), (1, 1, 16)):
        n = lib.fi_peer_gather_bytes(nbuf, rows, row_total)
        data = nbuf * rows * row_total
        assert 3 * data <= n <= 3 * data + 3 * 255 + 1024, (nbuf, rows, row_total, n)

    bases = (ctypes.c_void_p * 2)(None, None)
    pbases = ctypes.cast(bases, ctypes.POINTER(ctypes.c_void_p))

    def gather(src=None, rows=4, row_bytes=256, stride=256, world=2, rank=0, buffer=0, nbuf=2,
               max_rows=16, b=pbases):
        return lib.fi_peer_gather(src, rows, row_bytes, stride, b, world, rank, buffer, nbuf,
                                  max_rows, None, None)
    bad = _lib.FI_ERR_INVALID_ARG
    assert gather(world=0) == bad and gather(world=9) == bad
    assert gather(rank=2) == bad and gather(rank=-1) == bad
    assert gather(rows=17) == bad and gather(buffer=2) == bad and gather(nbuf=0) == bad
    # two or more ranks need two buffers: a rank one call ahead writes the other one
    assert gather(nbuf=1) == bad and "at least 2 buffers" in lib.fi_last_error().decode()
    assert gather(row_bytes=24) == _lib.FI_ERR_ALIGNMENT
    assert gather(stride=264) == _lib.FI_ERR_ALIGNMENT
    assert gather() == bad                      # null source rows
    assert gather(b=None) == bad                # no region table
    assert "fi_peer_gather" in lib.fi_last_error().decode()

    handle = ctypes.create_string_buffer(64)
    out = ctypes.c_void_p()
    assert lib.fi_peer_alloc(0, ctypes.byref(out), handle) == bad
    assert lib.fi_peer_alloc(1024, None, handle) == bad
    assert lib.fi_peer_open(None, ctypes.byref(out)) == bad
    assert lib.fi_peer_close(None) == _lib.FI_OK
    assert lib.fi_peer_free(None) == _lib.FI_OK


def test_peer_reduce_host_checks():
    """fi_small_gemm_peer_reduce's region size (one 704-byte slot per 16 outputs, per
    source rank and buffer, plus the local state) and the argument checks that answer
    before any device work, including two or more ranks with one buffer."""
    lib = _lib.load()
    assert lib.fi_peer_reduce_bytes(0, 2, 3072) == 0
    assert lib.fi_peer_reduce_bytes(2, 9, 3072) == 0
    assert lib.fi_peer_reduce_bytes(2, 2, 0) == 0
    for nbuf, world, n in ((28, 8, 3072), (2, 2, 100), (1, 1, 16)):
        items = -(-n // 16)
        assert lib.fi_peer_reduce_bytes(nbuf, world, n) == nbuf * world * items * 88 * 8 + 256
    s2 = _lib.strides(64, 1)
    bases = (ctypes.c_void_p * 2)(16, 16)
    pb = ctypes.cast(bases, ctypes.POINTER(ctypes.c_void_p))

    def call(x=16, w=16, c=16, m=4, n=64, k=64, world=2, rank=0, buffer=0, nbuf=2, flags=0, b=pb):
        return lib.fi_small_gemm_peer_reduce(x, w, c, None, m, n, k, s2, s2, s2, None, b, world,
                                             rank, buffer, nbuf, flags, None, None)
    bad = _lib.FI_ERR_INVALID_ARG
    assert call(world=0) == bad and call(world=9) == bad and call(rank=2) == bad
    assert call(buffer=2) == bad and call(nbuf=0) == bad
    assert call(nbuf=1) == bad and "at least 2 buffers" in lib.fi_last_error().decode()
    assert call(flags=4) == bad
    assert call(m=17) == _lib.FI_ERR_UNSUPPORTED
    assert call(k=100) == _lib.FI_ERR_UNSUPPORTED
    assert call(x=None) == bad and call(b=None) == bad
    assert call(x=8) == _lib.FI_ERR_ALIGNMENT


def test_norm_rope_varlen_host_checks():
    """fi_rms_norm, fi_rope_kv_write and fi_prefill_fwd_varlen reject bad sizes,
    unsupported shapes and null pointers before any device work, and treat empty
    inputs as no-ops."""
    lib = _lib.load()
    bad, unsup, ok = _lib.FI_ERR_INVALID_ARG, _lib.FI_ERR_UNSUPPORTED, _lib.FI_OK
    # rms_norm(x, weight, out, rows, hidden, x_row_stride, out_row_stride, eps, stream)
    assert lib.fi_rms_norm(None, None, None, -1, 3072, 3072, 3072, 1e-5, None) == bad
    assert lib.fi_rms_norm(None, None, None, 4, 3070, 3072, 3072, 1e-5, None) == unsup
    assert lib.fi_rms_norm(None, None, None, 0, 3072, 3072, 3072, 1e-5, None) == ok
    assert lib.fi_rms_norm(None, None, None, 4, 3072, 3072, 3072, 1e-5, None) == bad

    s2, s3, s4 = _lib.strides(1, 1), _lib.strides(1, 1, 1), _lib.strides(1, 1, 1, 1)

    def rope(batch=2, seq=3, nq=24, nkv=8, d=128, ptr=None):
        return lib.fi_rope_kv_write(ptr, batch, seq, nq, nkv, d, s4, ptr, ptr, 64, 128, None, 0,
                                    ptr, s4, None, None, ptr, ptr, ptr, 8, 64, 4, s4, s4, s2,
                                    None, None)
    assert rope(batch=-1) == bad and rope(nkv=0) == bad
    assert rope(d=100) == unsup
    assert rope(batch=0) == ok and rope(seq=0) == ok
    assert rope() == bad  # null pointers

    def varlen(batch=2, hq=24, hkv=8, max_s=128, total=200, d=128):
        return lib.fi_prefill_fwd_varlen(None, None, None, None, None, batch, hq, hkv, max_s,
                                         total, d, s3, s3, s3, s3, 0.1, None, None)
    assert varlen(batch=-1) == bad and varlen(hkv=0) == bad
    assert varlen(d=64) == unsup
    assert varlen(hq=24, hkv=7) == bad
    assert varlen(batch=0) == ok and varlen(total=0) == ok
    assert varlen() == bad  # null pointers
