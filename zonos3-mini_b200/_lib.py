"""ctypes binding of ``libzonos3_b200.so``, the C-ABI library every op of this package calls.

There is no fallback: when the library is missing or a call fails, the op raises. Status codes follow
``include/zonos3_b200.h``: 1 (invalid argument) raises ``ValueError``, every other non-zero status raises
``RuntimeError`` with the library's ``zb_last_error()`` message.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libzonos3_b200.so"

_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_u64 = ctypes.c_uint64

# name -> argument types (every entry point returns int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "zb_last_error": [],
    "zb_clear_error": [],
    "zb_version": [],
    "zb_launch_count": [],
    "zb_device_status": [_p, _i32],
    # q, k, v, q_stride_b, k_stride_b, v_stride_b, g, beta, gb_stride_b, state, slots, num_slots,
    # out, out_stride_b, B, H, dk, dv, scale, stream
    "zb_gdn_decode_step": [_p, _p, _p, _i64, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, _i64,
                           _i32, _i32, _i32, _i32, _f32, _p],
    # q, k, v, g, beta, cu_seqlens, num_seqs, H, dk, dv, scale, init_state, state_slots, final_state, out,
    # total_tokens, workspace, workspace_bytes, stream
    "zb_gdn_chunk_prefill": [_p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _f32, _p, _p, _p, _p, _i64, _p, _i64,
                             _p],
    # total_tokens, num_seqs, H, dk -> bytes (int64)
    "zb_gdn_chunk_prefill_workspace_bytes": [_i64, _i32, _i32, _i32],
    # mixed, mixed_stride, conv_weight, A_log, dt_bias, cu_seqlens, seq_of_token, slots, fresh, conv_state,
    # conv_rows, num_seqs, N, H, D, q, k, v, g, beta, stream
    "zb_gdn_prologue": [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p,
                        _p],
    # mixed, mixed_stride, conv_weight, A_log, dt_bias, slots, conv_state, conv_rows, N, H, D, q, k, v, g, beta,
    # stream
    "zb_gdn_prologue_decode": [_p, _i64, _p, _p, _p, _p, _p, _i64, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p],
    # ids, T, k, E, block, capacity, hist, counts, offsets, sorted_pairs, position, x, x_stride, D, x_perm, stream
    "zb_moe_permute_gather": [_p, _i32, _i32, _i32, _i32, _i64, _p, _p, _p, _p, _p, _p, _i64, _i32, _p, _p],
    # x_perm, capacity, gate_up, down, E, D, I, offsets, counts, sorted_pairs, weights, h, y, flags, stream
    "zb_moe_gemms": [_p, _i64, _p, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p],
    # T, N, K, block_n, splits -> bytes (int64)
    "zb_proj_gemm_workspace_bytes": [_i32, _i32, _i32, _i32, _i32],
    # x, x_stride, T, K, weight, N, out, out_stride, block_n, splits, workspace, workspace_bytes, stream
    "zb_proj_gemm": [_p, _i64, _i32, _i32, _p, _i32, _p, _i64, _i32, _i32, _p, _i64, _p],
    # x, x_stride, T, K, in_proj, conv_weight, A_log, dt_bias, slots, conv_state, conv_rows, H, D, q, k, v, z, g,
    # beta, splits, workspace, workspace_bytes, stream
    "zb_gdn_in_proj_decode": [_p, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p,
                              _i32, _p, _i64, _p],
    # o, z, z_stride, weight, eps, N, H, D, out, stream
    "zb_gdn_gated_norm": [_p, _p, _i64, _p, _f32, _i32, _i32, _i32, _p, _p],
    # bank, bank_stride, S, source, append, query, eps, norm_weight, norm_eps, out, mix_out, T, D, stream
    "zb_attnres_route": [_p, _i64, _i32, _p, _p, _p, _f32, _p, _f32, _p, _p, _p, _i64, _i32, _i32, _i32, _p],
    # bank, bank_stride, S, source, append, source_in_bank, queries, num_routes, route, eps, norm_weight, norm_eps,
    # out, mix_out, table, table_stride, inv_rms, inv_stride, T, D, stream
    "zb_attnres_route_tabled": [_p, _i64, _i32, _p, _p, _i32, _p, _i32, _i32, _f32, _p, _f32, _p, _p, _p, _i64, _p,
                                _i64, _i32, _i32, _p],
    # x, x_stride, norm_weight, eps, w_router, bias, T, D, E, k, weight_mode, renormalize, logits, ids, weights, stream
    "zb_moe_router": [_p, _i64, _p, _f32, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p, _p, _p],
    # logits, logits_bf16, bias, T, E, k, weight_mode, renormalize, ids, weights, stream
    "zb_moe_select": [_p, _i32, _p, _i32, _i32, _i32, _i32, _i32, _p, _p, _p],
    # ids, T, k, E, block, capacity, hist, counts, offsets, sorted_pairs, position, stream
    "zb_moe_permute": [_p, _i32, _i32, _i32, _i32, _i64, _p, _p, _p, _p, _p, _p],
    # x, x_stride, sorted_pairs, k, rows, D, out, stream
    "zb_moe_gather": [_p, _i64, _p, _i32, _i64, _i32, _p, _p],
    # x_perm, capacity, gate_up, E, D, I, offsets, h, stream
    "zb_moe_gemm_swiglu": [_p, _i64, _p, _i32, _i32, _i32, _p, _p, _p, _p],
    # h, capacity, down, E, D, I, offsets, sorted_pairs, weights, y, stream
    "zb_moe_gemm_down": [_p, _i64, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p],
    # y, T, k, D, out, out_stride, stream
    "zb_moe_combine": [_p, _i32, _i32, _i32, _p, _i64, _p],
    # h, capacity, down, E, D, I, offsets, counts, sorted_pairs, weights, T, k, out, out_stride, stream
    "zb_moe_down_combine_noalloc": [_p, _i64, _p, _i32, _i32, _i32, _p, _p, _p, _p, _i32, _i32, _p, _i64, _p],
    # k_cache, v_cache, slot_stride, num_slots, slots, k, k_stride, v, v_stride, N, Hkv, hd, stream
    "zb_kv_store": [_p, _p, _i64, _i64, _p, _p, _i64, _p, _i64, _i32, _i32, _i32, _p],
    # q, q_stride, k_cache, v_cache, slot_stride, num_slots, page_table, table_stride, seq_lens, max_seq_len, B, Hq,
    # Hkv, hd, scale, splits, split_len, workspace, workspace_bytes, out, out_stride, gate, gate_stride, stream
    # logits, logits_fp32, softcap, row_stride, batch_stride, B, C, V, temperatures, greedy, top_k, top_p, min_p, codebook_size, audio_pad_id,
    # stop_ids, codebook_sizes, stop_blocked, stop_bias, rep_ids, W, rep_penalties, seed, offset, offset_dev,
    # text_vocab, out, probs_out, stream
    "zb_sample_tts": [_p, _i32, _f32, _i64, _i64, _i32, _i32, _i32, _p, _i32, _i32, _f32, _f32, _i32, _i32, _p, _p, _p, _p, _p,
                      _i32, _p, _u64, _u64, _p, _i32, _p, _p, _p],
    # ids, ids_stride, ncols, tables (host array), table_rows (host array), norm_weight, eps, normalize, N, D, out,
    # out_stride, stream
    "zb_embed_norm": [_p, _i64, _i32, _p, _p, _p, _f32, _i32, _i32, _i32, _p, _i64, _p],
    # codes, codes_cols, ids, ids_cols, history, C, W, ring, counter, positions, seqlens, out_loc, page_table,
    # table_stride, max_len, B, stream
    "zb_decode_advance": [_p, _i32, _p, _i32, _p, _i32, _i32, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _p],
    # proj, proj_stride, temp, positions, theta, eps, q_out, k_cache, v_cache, slot_stride, num_slots, out_loc, N,
    # Hq, Hkv, hd, stream
    "zb_gqa_prologue_decode": [_p, _i64, _p, _p, _f32, _f32, _p, _p, _p, _i64, _i64, _p, _i32, _i32, _i32, _i32, _p],
    "zb_gqa_decode": [_p, _i64, _p, _p, _i64, _i64, _p, _i64, _p, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _p,
                      _i64, _p, _i64, _p, _i64, _p],
    # n, out (complex float64 [n]), stream
    "zb_istft_twiddles": [_i32, _p, _p],
    # y0, y0_stride, y1, y1_stride, y_is_f64, streams, cols, n0, n1, hop, window0, window1, twiddle0, twiddle1,
    # max_log_mag, mixer, taps, carry0, carry1, carry_parity, ring0, ring1, ring_size, frames_before, mix_from, mix_to,
    # flush, scratch, scratch_elems, out, stream
    "zb_istft_head_push": [_p, _i64, _p, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p, _p, _p, ctypes.c_double, _p, _i32,
                           _p, _p, _i32, _p, _p, _i32, _i64, _i64, _i64, _i32, _p, _i64, _p, _p],
    # x, x_is_f64, x_stride, streams, count, ring, ring_size, n_in_before, kernel_t, orig, new, width, block_from,
    # block_to, out_count, out, workspace, workspace_elems, stream
    "zb_resample_push": [_p, _i32, _i64, _i32, _i32, _p, _i32, _i64, _p, _i32, _i32, _i32, _i64, _i64, _i64, _p, _p,
                         _i64, _p],
}
_RESTYPES = {"zb_last_error": ctypes.c_char_p, "zb_clear_error": None, "zb_launch_count": ctypes.c_uint64,
             "zb_gdn_chunk_prefill_workspace_bytes": ctypes.c_int64, "zb_proj_gemm_workspace_bytes": ctypes.c_int64}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class LibraryMissing(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the library once and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise LibraryMissing(
                    f"{LIBRARY.name} is not built; run __graft_entry__.build() (nvcc, sm_100a) first"
                )
            lib = ctypes.CDLL(str(LIBRARY))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def launch_count() -> int:
    """Kernel launches the library has issued in this process (captured launches count once)."""
    return int(load().zb_launch_count())


def last_error() -> str:
    msg = load().zb_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status == 0:
        return
    msg = f"{what}: {last_error()} (status {status})"
    if status == 1:
        raise ValueError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    """Call entry point ``name`` and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)
