"""The allocation-free C entry point of the attention backward.

Some callers cannot allocate device memory (a host application that owns the
whole memory budget and hands a plugin fixed buffers; a latency-critical loop
that must not enter the CUDA allocator).  ``art_attn_bwd_noalloc`` serves
them: it takes every input and output from the caller and keeps its only
scratch in a fixed device array.  This test calls it through its exported C
symbol (ctypes) twice in a row and checks each result against the regular
``attn_bwd`` entry point.  It also checks every argument rule of the C
declaration (``art_noalloc.h``): each bad size, pointer, stride or alignment
is rejected with its return code before the device is touched.  The file name
sorts last so a run that stops at the first failure has run every other test
before this one.
"""

import ctypes
import math

import pytest
import torch

from art_mlx_b200.ops import fused, native
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_attn_bwd_noalloc_matches_entry_point(cuda):
    C = native.lib()
    lib = ctypes.CDLL(native.SO_PATH)
    fn = lib.art_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    i64, ptr = ctypes.c_int64, ctypes.c_void_p
    fn.argtypes = [ptr, i64, ptr, i64, ptr, i64, ptr, i64, ptr, i64, ptr, ptr, ptr, ctypes.c_int,
                   ptr, ptr, ptr, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ptr]

    torch.manual_seed(7)
    prompt = torch.randint(0, 1000, (150,))
    seqs = [torch.cat([prompt, torch.randint(0, 1000, (70,))]) for _ in range(4)]
    pack = prefix_tree_pack(seqs, max_depth=64, shareable_lengths=[149] * 4)
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    T, Hq, Hkv, D = kend.numel(), 4, 2, 128
    meta = fused.AttnMeta.build(torch.arange(T), kend, cuda)
    q = torch.randn(T, Hq, D, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(D)
    o, lse = C.attn_fwd(q, k, v, meta.kend, meta.tile_kmax, scale)
    do = torch.randn_like(o)
    units = fused.attention_bwd_units(kend).to(cuda)  # work units of the warp-level backward
    ref_dq, ref_dk, ref_dv = C.attn_bwd(do, q, k, v, o, lse, meta.kend, units, scale)

    dq = torch.full((T, Hq, D), 123.0, device=cuda)  # garbage: the entry point must clear it
    dk = torch.full((T, Hkv, D), -7.0, device=cuda)
    dv = torch.full((T, Hkv, D), 5.0, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        rc = fn(do.data_ptr(), do.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
                v.data_ptr(), v.stride(0), o.data_ptr(), o.stride(0), lse.data_ptr(), meta.kend.data_ptr(),
                units.data_ptr(), units.shape[0], dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                T, Hq, Hkv, D, scale, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call} returned {rc}"
        assert _rel(dq, ref_dq) < 2e-2
        assert _rel(dk, ref_dk) < 2e-2
        assert _rel(dv, ref_dv) < 2e-2

    def call(**over):
        a = dict(dout=do.data_ptr(), lddo=do.stride(0), q=q.data_ptr(), ldq=q.stride(0), k=k.data_ptr(),
                 ldk=k.stride(0), v=v.data_ptr(), ldv=v.stride(0), out=o.data_ptr(), ldo=o.stride(0),
                 lse=lse.data_ptr(), kend=meta.kend.data_ptr(), units=units.data_ptr(), n_units=units.shape[0],
                 dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), T=T, Hq=Hq, Hkv=Hkv, D=D)
        a.update(over)
        return fn(a["dout"], a["lddo"], a["q"], a["ldq"], a["k"], a["ldk"], a["v"], a["ldv"], a["out"], a["ldo"],
                  a["lse"], a["kend"], a["units"], a["n_units"], a["dq"], a["dk"], a["dv"], a["T"], a["Hq"],
                  a["Hkv"], a["D"], scale, stream)

    # rejected arguments return before anything touches the device
    assert call(T=1 << 20, Hq=2, Hkv=1) == 2  # beyond the fixed scratch
    assert call(D=64) == 3
    assert call(Hq=3) == 4  # Hq not a multiple of Hkv
    assert call(q=0) == 4  # null operand
    assert call(ldq=q.stride(0) + 4) == 4  # row stride not a multiple of 8 elements
    assert call(ldk=Hkv * D - 8) == 4  # row stride shorter than the row
    assert call(ldo=Hq * D - 8) == 4
    assert call(dout=do.data_ptr() + 2) == 4  # base not 16-byte aligned
    assert call(v=v.data_ptr() + 8) == 4
    assert call(dq=dq.data_ptr() + 4) == 4  # fp32 output not 16-byte aligned
    assert call(lse=0) == 4
    # the buffers are untouched by the rejected calls
    assert _rel(dq, ref_dq) < 2e-2
