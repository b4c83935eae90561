"""The C-ABI library, checked without a GPU: it loads, exports every entry point
include/ema_ssd_b200.h declares, and its host-side validation rejects bad
arguments before touching CUDA."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ema_ssd_b200.h")
SSD_HEADER = os.path.join(ROOT, "include", "ssd_b200.h")


def _declared():
    src = open(HEADER).read() + open(SSD_HEADER).read()
    return re.findall(r"EMA_API\s+[\w\s\*]+?\b(\w+)\s*\(", src)


def test_header_declares_entry_points():
    names = _declared()
    for n in ("ema_fwd_launch", "ema_bwd_launch", "chunk_cumsum_launch", "ema_scan_workspace_size",
              "ema_workspace_status", "ema_last_error", "ssd_fwd_launch", "ssd_bwd_launch", "ssd_internal_chunks"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from kernels import _lib
    for n in _declared():
        assert hasattr(_lib.lib, n), f"{n} not exported by {_lib._LIB_PATH}"


def test_struct_layouts_match_header():
    """ctypes mirrors of EmaFwdArgs / EmaBwdArgs have the C sizes (compiled with gcc here)."""
    import subprocess
    import tempfile
    from kernels import _lib
    code = ('#include "ema_ssd_b200.h"\n#include <stdio.h>\n#include <stddef.h>\n'
            'int main(){printf("%zu %zu %zu %zu\\n", sizeof(EmaFwdArgs), sizeof(EmaBwdArgs),'
            ' offsetof(EmaFwdArgs, workspace), offsetof(EmaBwdArgs, workspace));return 0;}\n')
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(code)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    sizes = [int(v) for v in out]
    assert sizes[0] == ctypes.sizeof(_lib.EmaFwdArgs)
    assert sizes[1] == ctypes.sizeof(_lib.EmaBwdArgs)
    assert sizes[2] == _lib.EmaFwdArgs.workspace.offset
    assert sizes[3] == _lib.EmaBwdArgs.workspace.offset


@pytest.mark.parametrize("header,struct", [("ema_ssd_b200.h", "EmaSpanFoldArgs"), ("ema_ssd_b200.h", "EmaSpanStateArgs"),
                                           ("ema_ssd_b200.h", "EmaSpanExchangeArgs"),
                                           ("ssd_b200.h", "SsdGateArgs")])
def test_every_field_offset_matches_header(header, struct):
    """The ctypes mirror of `struct` has the C size and every field at the C offset."""
    import subprocess
    import tempfile
    from kernels import _lib
    mirror = getattr(_lib, struct)
    fields = [f[0] for f in mirror._fields_]
    code = (f'#include "{header}"\n#include <stdio.h>\n#include <stddef.h>\nint main(){{printf("%zu'
            + ' %zu' * len(fields) + f'\\n", sizeof({struct})'
            + ''.join(f', offsetof({struct}, {f})' for f in fields) + ');return 0;}\n')
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(code)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        out = [int(v) for v in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(mirror)
    for k, f in enumerate(fields):
        assert out[1 + k] == getattr(mirror, f).offset, f


def test_ssd_struct_layouts_match_header():
    """ctypes mirrors of SsdFwdArgs / SsdBwdArgs have the C sizes and field offsets."""
    import subprocess
    import tempfile
    from kernels import _lib
    fields_f = ["final_state", "chunk_states", "out", "D", "dt_bias", "dt_softplus", "dt_clamp", "dt_min", "dt_max"]
    fields_b = ["d_initial_state", "dD", "ddt", "dout", "chunk_states", "dt_bias", "dt_softplus", "dt_clamp",
                "dt_min", "dt_max", "ddt_bias"]
    code = ('#include "ssd_b200.h"\n#include <stdio.h>\n#include <stddef.h>\nint main(){printf("%zu %zu'
            + ' %zu' * (len(fields_f) + len(fields_b)) + '\\n", sizeof(SsdFwdArgs), sizeof(SsdBwdArgs)'
            + ''.join(f', offsetof(SsdFwdArgs, {f})' for f in fields_f)
            + ''.join(f', offsetof(SsdBwdArgs, {f})' for f in fields_b) + ');return 0;}\n')
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(code)
        subprocess.run(["gcc", "-I", os.path.dirname(SSD_HEADER), c, "-o", exe], check=True)
        out = [int(v) for v in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(_lib.SsdFwdArgs)
    assert out[1] == ctypes.sizeof(_lib.SsdBwdArgs)
    for k, f in enumerate(fields_f):
        assert out[2 + k] == getattr(_lib.SsdFwdArgs, f).offset, f
    for k, f in enumerate(fields_b):
        assert out[2 + len(fields_f) + k] == getattr(_lib.SsdBwdArgs, f).offset, f


def test_ssd_validation_rejects_unsupported_shapes():
    """Host-side checks run before any device work (no GPU needed)."""
    from kernels import _lib
    a = _lib.SsdFwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.dstate, a.ngroups = 1, 64, 2, 32, 128, 1
    a.dtype = _lib.DTYPE_CODES[__import__("torch").bfloat16]
    assert _lib.lib.ssd_fwd_launch(a, None) == 2  # EMA_ERR_UNSUPPORTED: headdim 32
    assert b"headdim" in _lib.lib.ema_last_error()
    a.headdim, a.nheads, a.ngroups = 64, 3, 2
    assert _lib.lib.ssd_fwd_launch(a, None) == 1  # nheads not a multiple of ngroups
    assert _lib.lib.ssd_internal_chunks(4096) == 64 and _lib.lib.ssd_internal_chunks(65) == 2


def test_workspace_size_grows_with_tiles():
    from kernels import _lib
    f = _lib.lib.ema_scan_workspace_size
    small = f(1, 256, 1, 64, 256)
    big = f(8, 4096, 32, 64, 256)
    assert 256 < small < big
    assert big % 256 == 0


def _fwd_args(**kw):
    from kernels import _lib
    a = _lib.EmaFwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = 1, 256, 1, 64, 256
    a.dtype = 1
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code", [
    (dict(chunk_size=100), 2),          # unsupported chunk
    (dict(headdim=256), 2),             # headdim > 128
    (dict(headdim=60), 2),              # 120 bytes not a multiple of 16
    (dict(dtype=7), 1),                 # unknown dtype
    (dict(nheads=0), 1),                # bad shape
    (dict(), 1),                        # x / out missing
])
def test_forward_validation_without_gpu(kw, code):
    from kernels import _lib
    rc = _lib.lib.ema_fwd_launch(_fwd_args(**kw), None)
    assert rc == code, _lib.lib.ema_last_error()


def test_forward_needs_a_decay_and_a_workspace():
    from kernels import _lib
    fake = 1 << 20  # never dereferenced: validation fails first
    a = _fwd_args(x=fake, out=fake)
    assert _lib.lib.ema_fwd_launch(a, None) == 1  # neither dA nor dt/A
    a = _fwd_args(x=fake, out=fake, dA=fake, dt=fake, A=fake)
    assert _lib.lib.ema_fwd_launch(a, None) == 1  # both forms
    a = _fwd_args(x=fake, out=fake, dt=fake, A=fake, seq_idx=fake, seq_idx_type=2)
    assert _lib.lib.ema_fwd_launch(a, None) == 2  # seq_idx with the dt form
    a = _fwd_args(x=fake, out=fake, dA=fake)
    assert _lib.lib.ema_fwd_launch(a, None) == 3  # no workspace
    a = _fwd_args(x=fake, out=fake, dA=fake, workspace=fake, workspace_bytes=64)
    assert _lib.lib.ema_fwd_launch(a, None) == 3  # workspace too small
    assert b"workspace" in _lib.lib.ema_last_error()


def test_backward_validation_without_gpu():
    from kernels import _lib
    fake = 1 << 20
    a = _lib.EmaBwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size, a.dtype = 1, 256, 1, 64, 256, 1
    assert _lib.lib.ema_bwd_launch(a, None) == 1
    a.x = a.dout = a.dx = a.states = fake
    a.da_cs = fake
    assert _lib.lib.ema_bwd_launch(a, None) == 1  # dl output missing
    a.dl = fake
    assert _lib.lib.ema_bwd_launch(a, None) == 3  # workspace missing


def test_empty_problem_is_a_no_op():
    from kernels import _lib
    a = _fwd_args(seqlen=0)
    assert _lib.lib.ema_fwd_launch(a, None) == 0


def test_chunk_cumsum_validation_without_gpu():
    from kernels import _lib
    st = (_lib._i64 * 3)(1, 1, 1)
    assert _lib.lib.chunk_cumsum_launch(None, st, None, st, None, st, 1, 1, 1, 64, 0, None) == 1
    fake = 1 << 20
    assert _lib.lib.chunk_cumsum_launch(fake, st, fake, st, fake, st, 1, 1, 1, 2048, 0, None) == 2


def test_span_exchange_sizing_and_validation_without_gpu():
    """ema_span_exchange (the sequence-parallel exchange over NVLink peer
    memory): buffer sizing, and the argument checks that run before any CUDA
    call -- shape, rank, headdim, sub-span and buffer limits."""
    import ctypes
    from kernels import _lib
    L = _lib.lib
    assert L.ema_span_exchange_bytes(0, 32, 64) == 0 and L.ema_span_exchange_bytes(9, 32, 64) == 0
    n2, n4 = L.ema_span_exchange_bytes(2, 32, 64), L.ema_span_exchange_bytes(4, 32, 64)
    # header 256 + flags (8 ranks x 32 words, 256-aligned) + 2 parities x ranks x 32 x 65 floats
    assert n2 == 256 + 1024 + 2 * 2 * 32 * 65 * 4 and n4 == 256 + 1024 + 2 * 4 * 32 * 65 * 4

    def args(**kw):
        a = _lib.EmaSpanExchangeArgs()
        a.batch, a.subspans, a.nheads, a.headdim = 1, 8, 32, 64
        a.direction, a.rank, a.world = 0, 0, 2
        a.log_decay = a.values = a.span_in = a.out = 16  # never dereferenced: the checks fail first
        a.buffer_bytes = n2
        a.buffers[0] = a.buffers[1] = 16
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    cases = [(dict(headdim=256), 2, b"headdim"), (dict(subspans=65), 2, b"sub-spans"),
             (dict(rank=2), 1, b"rank"), (dict(world=9, rank=0), 1, b"rank"), (dict(direction=2), 1, b"direction"),
             (dict(values=None), 1, b"required"), (dict(buffer_bytes=n2 - 4), 3, b"buffers hold"),
             (dict(batch=0), 1, b"shape")]
    for kw, code, text in cases:
        assert L.ema_span_exchange(ctypes.byref(args(**kw)), None) == code, kw
        assert text in L.ema_last_error(), (kw, L.ema_last_error())
    assert L.ema_span_exchange(None, None) == 1
    assert L.ema_p2p_alloc(0, ctypes.byref(ctypes.c_void_p())) == 1
