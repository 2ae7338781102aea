"""The C ABI without a GPU: the library loads, exports every function include/nsa_sel.h declares,
and its host-side validation and launch planning behave (nothing here launches a kernel)."""
import ctypes
import subprocess

import pytest

from nsa_hopper_b200 import capi


def _desc(**kw):
    base = dict(q=256, k=256, v=256, sel=256, o=256, batch=1, heads_q=64, heads_kv=4, seq_len=65536, d_qk=128,
                d_v=128, n_qblocks=65536, n_sel=16, block_size=64, q_block=1)
    base.update(kw)
    return capi.make_desc(**base)


def test_library_exports_every_header_function():
    lib = capi.load()
    names = capi.header_functions()
    assert set(names) >= {"nsa_sel_forward", "nsa_sel_forward_lse", "nsa_sel_run", "nsa_sel_run_host", "nsa_sel_plan",
                          "nsa_sel_last_error", "nsa_sel_version"}
    for n in names:
        assert hasattr(lib, n), n
    assert lib.nsa_sel_version() == 10000


def test_struct_layout_matches_header(tmp_path):
    """The ctypes mirrors have the size and field offsets the C compiler gives the header's structs."""
    fields = [f for f, _ in capi.NsaSelDesc._fields_]
    pfields = [f for f, _ in capi.NsaSelPlanInfo._fields_]
    hfields = [f for f, _ in capi.NsaSelHostIO._fields_]
    bfields = [f for f, _ in capi.NsaSelBwdDesc._fields_]
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{capi.HEADER_PATH}"', "int main(void) {",
             'printf("%zu\\n", sizeof(nsa_sel_desc));', 'printf("%zu\\n", sizeof(nsa_sel_plan_info));',
             'printf("%zu\\n", sizeof(nsa_sel_host_io));', 'printf("%zu\\n", sizeof(nsa_sel_bwd_desc));']
    lines += [f'printf("%zu\\n", offsetof(nsa_sel_desc, {f}));' for f in fields]
    lines += [f'printf("%zu\\n", offsetof(nsa_sel_plan_info, {f}));' for f in pfields]
    lines += [f'printf("%zu\\n", offsetof(nsa_sel_host_io, {f}));' for f in hfields]
    lines += [f'printf("%zu\\n", offsetof(nsa_sel_bwd_desc, {f}));' for f in bfields]
    lines += ["return 0; }"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(capi.NsaSelDesc) and vals[1] == ctypes.sizeof(capi.NsaSelPlanInfo)
    assert vals[2] == ctypes.sizeof(capi.NsaSelHostIO) and vals[3] == ctypes.sizeof(capi.NsaSelBwdDesc)
    got = vals[4:]
    want = [getattr(capi.NsaSelDesc, f).offset for f in fields] + [getattr(capi.NsaSelPlanInfo, f).offset for f in pfields]
    want += [getattr(capi.NsaSelHostIO, f).offset for f in hfields]
    want += [getattr(capi.NsaSelBwdDesc, f).offset for f in bfields]
    assert got == want


def test_plan_north_star():
    p = capi.plan(_desc())
    assert p["n_cols"] == 16 and p["q_per_unit"] == 1 and p["parts"] == 1
    assert p["n_units"] == 4 * 65536 and p["grid"] == 148
    assert p["smem_bytes"] <= 232448 and p["k_stages"] >= 2 and p["v_stages"] >= 2


def test_plan_query_block_mode_splits_wide_groups():
    kw = dict(heads_q=16, heads_kv=1, seq_len=768, n_qblocks=48, n_sel=6, d_qk=64, d_v=64, q_block=16,
              o_dtype=capi.DTYPE_F32)
    # G = 16 with BQ = 16 is 256 query rows: two 128-row units for the row-owner kernel
    p = capi.plan(_desc(**kw))
    assert p["n_cols"] == 128 and p["q_per_unit"] == 8 and p["parts"] == 2 and p["n_units"] == 48 * 2
    assert p["tmem_cols"] == 512 and p["smem_bytes"] <= 232448
    # without it (debug flag NSA_DEBUG_NO_ROW_OWNER): parts of 4 tokens (N = 64) for the swap-AB kernel
    p = capi.plan(_desc(debug_flags=capi.NSA_DEBUG_NO_ROW_OWNER, **kw))
    assert p["n_cols"] == 64 and p["q_per_unit"] == 4 and p["parts"] == 4 and p["n_units"] == 48 * 4


def test_plan_row_owner_tiles():
    # BQ * G = 64 (the reference's own mode): a 64-row tile of the row-owner kernel (zero padded)
    p = capi.plan(_desc(heads_q=32, heads_kv=2, q_block=4, n_qblocks=16384, o_dtype=capi.DTYPE_F32))
    assert p["n_cols"] == 128 and p["q_per_unit"] == 4
    # G = 128 takes one token per tile; BQ * G = 32 stays on the swap-AB kernel
    p = capi.plan(_desc(heads_q=128, heads_kv=1))
    assert p["n_cols"] == 128 and p["q_per_unit"] == 1
    assert capi.plan(_desc(heads_q=32, heads_kv=4, q_block=4, n_qblocks=16384))["n_cols"] == 32
    # the reference op's cycle counters do not change the kernel: both kernels fill them
    assert capi.plan(_desc(q_block=8, n_qblocks=8192, cyc=256))["n_cols"] == 128
    assert capi.plan(_desc(heads_q=128, heads_kv=1, cyc=256))["n_cols"] == 128


def test_plan_small_group_pads_columns():
    p = capi.plan(_desc(heads_q=32, heads_kv=8))  # G = 4 -> one N=16 tile per token
    assert p["n_cols"] == 16


@pytest.mark.parametrize("kw,code", [
    (dict(q=0), capi.NSA_ERR_INVALID_ARG),
    (dict(q=258), capi.NSA_ERR_INVALID_ARG),               # TMA needs 16-byte aligned bases
    (dict(heads_q=63), capi.NSA_ERR_INVALID_ARG),          # Hq % Hkv != 0
    (dict(n_qblocks=100), capi.NSA_ERR_INVALID_ARG),       # NQB != ceil(T/BQ)
    (dict(block_size=96), capi.NSA_ERR_UNSUPPORTED),
    (dict(d_qk=96), capi.NSA_ERR_UNSUPPORTED),
    (dict(o_dtype=7), capi.NSA_ERR_INVALID_ARG),
    (dict(cu_seqlens=256, batch=2, n_qblocks=65536), capi.NSA_ERR_INVALID_ARG),
    (dict(bkv_begin=3, bkv_end=2), capi.NSA_ERR_INVALID_ARG),
    (dict(qb_begin=70000), capi.NSA_ERR_INVALID_ARG),
    (dict(n_sel=200), capi.NSA_ERR_UNSUPPORTED),           # more than 128 sub-blocks per unit
])
def test_validation_errors(kw, code):
    with pytest.raises(capi.NsaSelError) as e:
        capi.plan(_desc(**kw))
    assert e.value.code == code
    assert capi.last_error() != ""


def test_shard_plan_counts_units():
    p = capi.plan(_desc(bkv_begin=1, bkv_end=3, qb_begin=100, qb_end=1100))
    assert p["n_units"] == 2 * 1000


@pytest.mark.parametrize("args,code", [
    (dict(q=0), capi.NSA_ERR_INVALID_ARG),
    (dict(workspace=264), capi.NSA_ERR_INVALID_ARG),          # workspace must be 16-byte aligned
    (dict(Hq=7), capi.NSA_ERR_INVALID_ARG),                   # Hq % Hkv != 0
    (dict(d=68), capi.NSA_ERR_UNSUPPORTED),                   # d % 8 != 0
    (dict(q=258), capi.NSA_ERR_INVALID_ARG),                  # q must be 16-byte aligned
    (dict(d=512), capi.NSA_ERR_UNSUPPORTED),                  # d > 256
    (dict(n_sel=40), capi.NSA_ERR_UNSUPPORTED),               # top-k > 32
    (dict(l_prime=0), capi.NSA_ERR_INVALID_ARG),
])
def test_select_validation_errors(args, code):
    a = dict(q=256, k=256, workspace=256, sel=256, B=1, Hq=8, Hkv=2, T=4096, d=128, l_prime=64, n_sel=16)
    a.update(args)
    lib = capi.load()
    rc = lib.nsa_sel_select(ctypes.c_void_p(a["q"]), ctypes.c_void_p(a["k"]), ctypes.c_void_p(a["workspace"]),
                            ctypes.c_void_p(a["sel"]), a["B"], a["Hq"], a["Hkv"], a["T"], a["d"], a["l_prime"],
                            a["n_sel"], 32, 16, None)
    assert rc == code, capi.last_error()


def test_select_workspace_bytes():
    assert capi.select_workspace_bytes(1, 4, 65536, 128, 64) == 4 * 1024 * 128 * 4
    assert capi.select_workspace_bytes(2, 2, 500, 64, 64) == 2 * 2 * 8 * 64 * 4
    assert capi.select_workspace_bytes(0, 2, 500, 64, 64) == -1


@pytest.mark.parametrize("kw,code", [
    (dict(kv_len=-1), capi.NSA_ERR_INVALID_ARG),
    (dict(window=-5), capi.NSA_ERR_INVALID_ARG),
    (dict(key_map=2), capi.NSA_ERR_INVALID_ARG),
    (dict(kv_len=4095), capi.NSA_ERR_INVALID_ARG),                        # kv_len != T needs the compressed map
    (dict(kv_len=4095, key_map=1, window=64), capi.NSA_ERR_UNSUPPORTED),  # window + compressed map
    (dict(window=64, cu_seqlens=256, n_seqs=1), capi.NSA_ERR_UNSUPPORTED),
])
def test_key_visibility_validation(kw, code):
    with pytest.raises(capi.NsaSelError) as e:
        capi.plan(_desc(**kw))
    assert e.value.code == code


def test_compressed_key_map_plan():
    p = capi.plan(_desc(kv_len=4095, key_map=1, n_sel=64, o_dtype=capi.DTYPE_F32))
    assert p["n_units"] == 4 * 65536


def test_extended_visibility_needs_fp32_variant():
    with pytest.raises(capi.NsaSelError) as e:
        capi.plan(_desc(window=512))  # bf16 O: no window variant is built
    assert e.value.code == capi.NSA_ERR_UNSUPPORTED
    assert capi.plan(_desc(window=512, o_dtype=capi.DTYPE_F32))["n_cols"] == 16


@pytest.mark.parametrize("kw,code", [
    (dict(o_accumulate=1), capi.NSA_ERR_UNSUPPORTED),                   # bf16 O cannot be accumulated
    (dict(o_accumulate=2, o_dtype=capi.DTYPE_F32), capi.NSA_ERR_INVALID_ARG),
    (dict(o_weight=258, o_dtype=capi.DTYPE_F32), capi.NSA_ERR_INVALID_ARG),  # misaligned weight pointer
])
def test_fused_output_validation(kw, code):
    with pytest.raises(capi.NsaSelError) as e:
        capi.plan(_desc(**kw))
    assert e.value.code == code


def test_fused_output_plan():
    p = capi.plan(_desc(o_accumulate=1, o_weight=260, o_dtype=capi.DTYPE_F32))
    assert p["n_cols"] == 16


def test_host_path_validation():
    """nsa_sel_run_host rejects bad host descriptions before touching the GPU (no device here:
    the device query fails after the argument checks, so only argument errors are asserted)."""
    lib = capi.load()
    d = _desc(o_dtype=capi.DTYPE_F32, o_accumulate=1)
    io = capi.make_host_io(q=256, k=256, v=256, sel=256, o=256)
    assert lib.nsa_sel_run_host(ctypes.byref(d), None, None) == capi.NSA_ERR_INVALID_ARG
    assert lib.nsa_sel_run_host(ctypes.byref(d), ctypes.byref(capi.make_host_io(q=256)), None) == capi.NSA_ERR_INVALID_ARG
    assert lib.nsa_sel_run_host(ctypes.byref(d), ctypes.byref(io), None) == capi.NSA_ERR_UNSUPPORTED
    io.token_slices = -1
    assert lib.nsa_sel_run_host(ctypes.byref(_desc()), ctypes.byref(io), None) == capi.NSA_ERR_INVALID_ARG


def _bwd(**kw):
    base = dict(q=16, k=16, v=16, sel=16, o=16, lse=16, d_o=16, dq=16, dk=16, dv=16, workspace=16, batch=1,
                heads_q=64, heads_kv=4, seq_len=65536, d=128, n_sel=16, block_size=64)
    base.update(kw)
    return capi.make_bwd_desc(**base)


def test_backward_workspace_bytes():
    """Row sums (B*Hq*T floats) + index: 4 bucket arrays, token entries (B*Hkv*T*KSEL*l'/64 at
    most) and 16-byte work items, each region 16-byte aligned.  A bucket is (b*Hkv + kvh, token
    window, 64-key sub-block): 4096-token windows for G = 16 at T = 64K."""
    n = capi.backward_workspace_bytes(_bwd())
    rows, buckets, pairs = 64 * 65536, 4 * 16 * 1024, 4 * 65536 * 16
    expect = rows * 4 + 3 * buckets * 4 + (buckets + 1) * 4 + pairs * 4 + (pairs // 128 + buckets) * 16
    assert expect <= n <= expect + 7 * 16
    assert capi.backward_workspace_bytes(_bwd(block_size=128, n_sel=4)) < n


@pytest.mark.parametrize("Hq, Hkv, T, n_win", [
    (64, 8, 65536, 8),      # G = 8: 8192-token windows
    (64, 4, 4096, 1),       # one window
    (64, 4, 1 << 20, 32),   # long sequences: at most 32 windows (32768 tokens each)
    (64, 4, 4097, 2),       # a partial last window
])
def test_backward_workspace_counts_token_windows(Hq, Hkv, T, n_win):
    """The inverse index has one bucket per (b*Hkv + kvh, token window, 64-key sub-block)."""
    n = capi.backward_workspace_bytes(_bwd(heads_q=Hq, heads_kv=Hkv, seq_len=T, n_sel=4))
    nsub = (T + 63) // 64
    rows, buckets, pairs = Hq * T, Hkv * n_win * nsub, Hkv * T * min(4, nsub)
    expect = rows * 4 + 3 * buckets * 4 + (buckets + 1) * 4 + pairs * 4 + (pairs // 128 + buckets) * 16
    assert expect <= n <= expect + 7 * 16


@pytest.mark.parametrize("kw, code", [
    (dict(heads_q=32, heads_kv=8), capi.NSA_ERR_UNSUPPORTED),   # G = 4
    (dict(d=64), capi.NSA_ERR_UNSUPPORTED),
    (dict(block_size=96), capi.NSA_ERR_UNSUPPORTED),
    (dict(heads_q=65), capi.NSA_ERR_INVALID_ARG),
    (dict(n_sel=0), capi.NSA_ERR_INVALID_ARG),
    (dict(o_dtype=7), capi.NSA_ERR_INVALID_ARG),
])
def test_backward_validation(kw, code):
    """The description is checked before any device call (this runs without a GPU)."""
    with pytest.raises(capi.NsaSelError) as ei:
        capi.backward(_bwd(**kw))
    assert ei.value.code == code
    with pytest.raises(capi.NsaSelError):  # the size query reports -1 for the same descriptions
        capi.backward_workspace_bytes(_bwd(**kw))


def test_backward_rejects_null_and_misaligned_pointers_before_touching_a_device():
    with pytest.raises(capi.NsaSelError) as ei:
        capi.backward(_bwd(dq=None))
    assert ei.value.code == capi.NSA_ERR_INVALID_ARG
    with pytest.raises(capi.NsaSelError) as ei:
        capi.backward(_bwd(dk=24))
    assert ei.value.code == capi.NSA_ERR_INVALID_ARG


def test_torch_backward_checks_its_tensors_before_any_device_call():
    """ops.backward refuses host tensors and wrong dtypes with a ValueError (no GPU needed)."""
    import torch

    from nsa_hopper_b200 import ops

    q = torch.zeros(1, 16, 64, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 64, 128, dtype=torch.bfloat16)
    sel = torch.zeros(1, 2, 64, 1, dtype=torch.int32)
    lse = torch.zeros(1, 16, 64)
    with pytest.raises(ValueError, match="Q must be a contiguous bf16 CUDA tensor"):
        ops.backward(q, k, k, sel, q, lse, q)
    with pytest.raises(ValueError, match="Q must be"):
        ops.backward(q.float(), k, k, sel, q, lse, q)
