"""wohper_b200 -- B200 (sm_100a) dequant-matmul hot path of Wohper.

This package is the Python host side of the C ABI declared in
``include/wohper_b200.h`` (library ``wohper_b200/libwohper_b200.so``).  Its
functions carry the names of the reference engine's Rust functions they stand
in for (engine/zc_infer_core), take torch CUDA tensors (device memory), run
asynchronously on the current torch stream, and raise :class:`WohperError`
with the reference's error kind (``DeepSeekV4KernelError`` order) on failure.

There is no CPU fallback: if the CUDA library is missing or the device is not
an sm_100 part, every call raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

from . import build as _build

HERE = Path(__file__).resolve().parent
LIB_PATH = _build.LIB

STATUS_NAMES = {
    0: "Ok",
    1: "EmptyShape",
    2: "InvalidShape",
    3: "PackedWeightTooSmall",
    4: "ScaleTooSmall",
    5: "InputTooSmall",
    6: "OutputTooSmall",
    7: "ScratchTooSmall",
    8: "NonFiniteOutput",
    9: "InvalidPointer",
    10: "Unsupported",
    20: "Cuda",
    21: "Nccl",
    22: "Timeout",
    23: "DeviceArg",
    30: "InvalidQuantBlockMagic",
    31: "UnsupportedQuantBlockVersion",
    32: "TruncatedQuantBlock",
    33: "InvalidQuantBlock",
    34: "TensorIndexOutOfRange",
    40: "Io",
    41: "InvalidMagic",
    42: "UnsupportedVersion",
    43: "Unaligned",
    44: "TruncatedManifest",
    45: "LayerCountMismatch",
    46: "InvalidExpertTable",
    47: "ShardMap",
    48: "InvalidExpert",
}
ROUTER_RAW_LOGITS = 0
ROUTER_SQRT_SOFTPLUS = 1
# wh_moe_scratch_field fields (include/wohper_b200.h)
MOE_FIELD_SLOT, MOE_FIELD_OFFSETS, MOE_FIELD_COMBINE_W = 1, 2, 3
MOE_FIELD_XQ, MOE_FIELD_XSF, MOE_FIELD_HQ, MOE_FIELD_HSF, MOE_FIELD_YROWS = 4, 5, 6, 7, 8

# Every symbol include/wohper_b200.h declares (checked by tests/test_capi.py).
EXPORTS = (
    "wh_version", "wh_ctx_create", "wh_ctx_destroy", "wh_ctx_sync", "wh_last_error_detail",
    "wh_fp8_gemv", "wh_act_quant_fp8", "wh_fp4_matvec", "wh_fp4_expert_scratch_len",
    "wh_fp4_expert_forward", "wh_router_topk", "wh_moe_plan_create", "wh_moe_plan_destroy",
    "wh_moe_scratch_bytes", "wh_moe_scratch_field", "wh_moe_ffn", "wh_debug_act_quant_table",
    "wh_debug_e4m3_round",
    "wh_ctx_set_profiling", "wh_ctx_phase_times", "wh_debug_e4m3_round_n",
    "wh_fp4_expert_forward_noalloc", "wh_ep_row_bytes", "wh_ep_scratch_bytes", "wh_ep_dispatch",
    "wh_ep_expert_ffn", "wh_ep_combine", "wh_ep_window_bytes", "wh_ep_window_create",
    "wh_ep_window_connect", "wh_ep_window_destroy", "wh_ep_p2p_dispatch",
    "wh_ep_p2p_expert_ffn", "wh_ep_p2p_combine", "wh_ep_moe_layer",
    "wh_moe_plan_set_fused_decode",
    "wh_zcblk_parse", "wh_zcblk_tensor_at", "wh_zcblk_tensor_dim", "wh_zcblk_find_suffix",
    "wh_zcblk_fp4_expert", "wh_fp4_expert_device_bytes", "wh_fp4_expert_upload",
    "wh_model_open", "wh_model_close", "wh_model_get_header", "wh_model_layer_count",
    "wh_model_get_layer", "wh_model_get_expert", "wh_model_expert_source",
    "wh_expert_loader_create", "wh_expert_loader_destroy", "wh_expert_arena_bytes",
    "wh_expert_loader_load", "wh_lm_head_scratch_bytes", "wh_lm_head_topk",
    "wh_fp8_expert_scratch_len", "wh_fp8_expert_forward", "wh_rope_inv_freqs",
    "wh_mla_attention", "wh_debug_expf_table", "wh_debug_expf_near", "wh_debug_ref_expf", "wh_hc_pre",
    "wh_hc_post", "wh_hc_head", "wh_rms_norm", "wh_fp8_gemv_grouped",
    "wh_v4_attention_scratch_len", "wh_v4_attention", "wh_lm_head_batch_scratch_bytes",
    "wh_lm_head_topk_batch",
)


class WohperError(RuntimeError):
    def __init__(self, status: int, detail: str = ""):
        self.status = status
        self.kind = STATUS_NAMES.get(status, f"Status{status}")
        super().__init__(f"{self.kind} ({status}): {detail}")


class Fp4MatvecSpec(C.Structure):
    """wh_fp4_matvec_spec == Fp4Matvec (src/deepseek_v4.rs:410-417)."""
    _fields_ = [
        ("packed_weight", C.c_void_p), ("packed_len", C.c_size_t),
        ("ue8m0_scales", C.c_void_p), ("scales_len", C.c_size_t),
        ("rows", C.c_size_t), ("cols", C.c_size_t), ("scale_cols", C.c_size_t),
    ]


class Fp4ExpertSpec(C.Structure):
    """wh_fp4_expert == DeepSeekV4Fp4Expert (src/deepseek_v4.rs:419-428)."""
    _fields_ = [("w1", Fp4MatvecSpec), ("w3", Fp4MatvecSpec), ("w2", Fp4MatvecSpec)]


class Fp8MatrixSpec(C.Structure):
    """wh_fp8_matrix: E4M3 weight [rows][cols] + UE8M0 scales [scale_rows][scale_cols]."""
    _fields_ = [("weight", C.c_void_p), ("scale", C.c_void_p), ("rows", C.c_int),
                ("cols", C.c_int), ("scale_rows", C.c_int), ("scale_cols", C.c_int)]


class Fp8ExpertSpec(C.Structure):
    """wh_fp8_expert: DeepSeek-V4's FP8 shared expert (w1, w3, w2)."""
    _fields_ = [("w1", Fp8MatrixSpec), ("w3", Fp8MatrixSpec), ("w2", Fp8MatrixSpec)]


class MoeDesc(C.Structure):
    _fields_ = [
        ("num_experts", C.c_int), ("hidden", C.c_int), ("inter", C.c_int),
        ("experts", C.POINTER(Fp4ExpertSpec)), ("shared", C.POINTER(Fp4ExpertSpec)),
        ("gate", C.c_void_p), ("gate_bias", C.c_void_p), ("topk", C.c_int),
        ("router_mode", C.c_int), ("route_scale", C.c_float), ("max_tokens", C.c_int),
        ("exact", C.c_int), ("shared_fp8", C.POINTER(Fp8ExpertSpec)),
    ]


_lib: Optional[C.CDLL] = None


def lib(build_if_missing: bool = True) -> C.CDLL:
    """Load libwohper_b200.so (building it first if asked and it is stale)."""
    global _lib
    if _lib is not None:
        return _lib
    if build_if_missing and not _build.up_to_date():
        _build.build()
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run python -m wohper_b200.build")
    L = C.CDLL(str(LIB_PATH))
    vp, i, sz, f = C.c_void_p, C.c_int, C.c_size_t, C.c_float
    st = C.c_int
    sig = {
        "wh_version": (i, []),
        "wh_ctx_create": (st, [i, C.POINTER(vp)]),
        "wh_ctx_destroy": (None, [vp]),
        "wh_ctx_sync": (st, [vp, vp]),
        "wh_last_error_detail": (C.c_char_p, []),
        "wh_fp8_gemv": (st, [vp, vp, vp, i, i, i, i, i, i, vp, i, i, vp, i, i, vp]),
        "wh_act_quant_fp8": (st, [vp, vp, sz, i, vp]),
        "wh_fp4_matvec": (st, [vp, C.POINTER(Fp4MatvecSpec), vp, sz, vp, sz, vp]),
        "wh_fp4_expert_scratch_len": (sz, [sz]),
        "wh_fp4_expert_forward": (st, [vp, C.POINTER(Fp4ExpertSpec), vp, sz, vp, sz, vp, sz, vp]),
        "wh_fp4_expert_forward_noalloc": (st, [vp, C.POINTER(Fp4ExpertSpec), vp, sz, vp, sz, vp]),
        "wh_ep_row_bytes": (sz, [i]),
        "wh_ep_scratch_bytes": (sz, [vp, i, i, i]),
        "wh_ep_dispatch": (st, [vp, vp, i, vp, i, vp, vp, vp, vp, vp, sz, vp]),
        "wh_ep_expert_ffn": (st, [vp, vp, i, vp, vp, i, vp, i, vp, vp, sz, vp]),
        "wh_ep_combine": (st, [vp, vp, vp, vp, vp, i, vp, vp, vp, vp]),
        "wh_ep_window_bytes": (sz, [vp, i, i]),
        "wh_ep_window_create": (st, [vp, vp, i, i, i, C.POINTER(vp), vp]),
        "wh_ep_window_connect": (st, [vp, vp]),
        "wh_ep_window_destroy": (None, [vp]),
        "wh_ep_p2p_dispatch": (st, [vp, vp, vp, i, vp, vp, vp]),
        "wh_ep_p2p_expert_ffn": (st, [vp, vp, vp, i, vp, vp]),
        "wh_ep_p2p_combine": (st, [vp, vp, vp, vp, vp, i, vp, vp, vp]),
        "wh_ep_moe_layer": (st, [vp, vp, vp, i, vp, vp, vp, vp]),
        "wh_router_topk": (st, [vp, vp, i, i, vp, i, i, i, vp, f, vp, vp, vp, vp, vp]),
        "wh_moe_plan_create": (st, [vp, C.POINTER(MoeDesc), C.POINTER(vp)]),
        "wh_moe_plan_destroy": (None, [vp]),
        "wh_moe_plan_set_fused_decode": (st, [vp, i]),
        "wh_moe_scratch_bytes": (sz, [vp, i]),
        "wh_rms_norm": (st, [vp, vp, vp, i, i, vp, vp]),
        "wh_fp8_gemv_grouped": (st, [vp, vp, vp, i, i, i, i, i, i, vp, i, i, i, C.c_longlong, vp,
                                     i, i, vp]),
        "wh_v4_attention_scratch_len": (sz, [vp, i]),
        "wh_v4_attention": (st, [vp, vp, i, vp, vp, vp, i, vp, vp, vp, vp, sz, vp]),
        "wh_moe_scratch_field": (st, [vp, i, i, C.POINTER(sz), C.POINTER(sz)]),
        "wh_moe_ffn": (st, [vp, vp, vp, i, vp, vp, vp, vp, vp, sz, vp]),
        "wh_debug_act_quant_table": (None, [vp]),
        "wh_debug_e4m3_round": (f, [f]),
        "wh_debug_e4m3_round_n": (None, [vp, vp, sz]),
        "wh_ctx_set_profiling": (st, [vp, i]),
        "wh_ctx_phase_times": (i, [vp, vp, i]),
        "wh_lm_head_scratch_bytes": (sz, [C.c_longlong, i]),
        "wh_rope_inv_freqs": (None, [i, f, f, f, f, C.c_uint64, vp]),
        "wh_debug_expf_table": (i, [C.POINTER(vp), C.POINTER(vp)]),
        "wh_debug_expf_near": (C.c_double, []),
        "wh_debug_ref_expf": (st, [vp, vp, vp, sz, vp]),
        "wh_hc_pre": (st, [vp, vp, vp, vp, vp, i, i, i, i, f, vp, vp, vp, vp]),
        "wh_hc_post": (st, [vp, vp, vp, vp, vp, i, i, i, vp, vp]),
        "wh_hc_head": (st, [vp, vp, f, vp, vp, i, i, i, f, vp, vp]),
        "wh_mla_attention": (st, [vp, vp, i, i, i, vp, i, i, i, vp, i, vp, vp, vp, vp]),
        "wh_fp8_expert_scratch_len": (sz, [sz, sz]),
        "wh_fp8_expert_forward": (st, [vp, C.POINTER(Fp8ExpertSpec), vp, sz, vp, sz, vp, sz,
                                       vp]),
        "wh_lm_head_topk": (st, [vp, vp, C.c_longlong, i, C.c_uint32, vp, sz, i, vp, vp, vp, vp,
                                 sz, vp]),
        "wh_lm_head_batch_scratch_bytes": (sz, [C.c_longlong, i, i]),
        "wh_lm_head_topk_batch": (st, [vp, vp, C.c_longlong, i, C.c_uint32, vp, i, i, i, vp, vp,
                                       vp, vp, sz, vp]),
        "wh_zcblk_parse": (st, [vp, sz, vp]),
        "wh_zcblk_tensor_at": (st, [vp, sz, C.c_uint32, vp]),
        "wh_zcblk_tensor_dim": (st, [vp, sz, vp, C.c_uint32, vp]),
        "wh_zcblk_find_suffix": (st, [vp, sz, C.c_char_p, vp]),
        "wh_zcblk_fp4_expert": (st, [vp, sz, vp]),
        "wh_fp4_expert_device_bytes": (sz, [C.c_uint64]),
        "wh_fp4_expert_upload": (st, [vp, vp, sz, vp, sz, C.POINTER(Fp4ExpertSpec), vp]),
        "wh_model_open": (st, [C.c_char_p, i, C.POINTER(vp)]),
        "wh_model_close": (None, [vp]),
        "wh_model_get_header": (st, [vp, vp]),
        "wh_model_layer_count": (i, [vp]),
        "wh_model_get_layer": (st, [vp, i, vp]),
        "wh_model_get_expert": (st, [vp, i, i, vp]),
        "wh_model_expert_source": (st, [vp, i, C.c_uint32, vp]),
        "wh_expert_loader_create": (st, [vp, vp, i, i, C.POINTER(vp)]),
        "wh_expert_loader_destroy": (None, [vp]),
        "wh_expert_arena_bytes": (st, [vp, i, vp, i, C.POINTER(sz)]),
        "wh_expert_loader_load": (st, [vp, i, vp, i, vp, sz, C.POINTER(Fp4ExpertSpec), vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(status: int) -> None:
    if status != 0:
        detail = lib().wh_last_error_detail()
        raise WohperError(status, detail.decode() if detail else "")


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    return int(t.data_ptr())


def _stream(stream=None) -> Optional[int]:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


class Context:
    """wh_ctx: one per device; owns the device status word."""

    def __init__(self, device: int = 0):
        import torch

        if not torch.cuda.is_available():
            raise RuntimeError("wohper_b200 needs a CUDA device (sm_100a); none is visible")
        torch.cuda.set_device(device)
        self.device = device
        h = C.c_void_p()
        _check(lib().wh_ctx_create(device, C.byref(h)))
        self.handle = h

    def sync(self, stream=None) -> None:
        """Synchronise and raise the first device-side error (NonFiniteOutput...)."""
        _check(lib().wh_ctx_sync(self.handle, _stream(stream)))

    def set_profiling(self, on: bool) -> None:
        _check(lib().wh_ctx_set_profiling(self.handle, int(bool(on))))

    def phase_times(self, max_phases: int = 16) -> list:
        buf = (C.c_float * max_phases)()
        n = lib().wh_ctx_phase_times(self.handle, C.cast(buf, C.c_void_p), max_phases)
        return [float(buf[i]) for i in range(n)]

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().wh_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------
# FP8 GEMV family (src/compute.rs:6174-6577)
# --------------------------------------------------------------------------
def gemv_fp8_e4m3_ue8m0_rows_multi(ctx: Context, weight, scale, inputs, row_start: int,
                                   row_end: int, outputs=None, act_quant_block: int = 0,
                                   stream=None):
    """Batched row-range FP8 GEMV: outputs[b, r-row_start] for rows [row_start,row_end)."""
    import torch

    rows, cols = weight.shape
    srows, scols = scale.shape
    if inputs.dim() == 1:
        inputs = inputs.view(1, -1)
    batch = inputs.shape[0]
    if outputs is None:
        outputs = torch.empty(batch, row_end - row_start, device=inputs.device, dtype=torch.float32)
    _check(lib().wh_fp8_gemv(ctx.handle, _ptr(weight), _ptr(scale), rows, cols, srows, scols,
                             row_start, row_end, _ptr(inputs), batch, inputs.stride(0),
                             _ptr(outputs), outputs.stride(0) if outputs.dim() > 1 else outputs.numel(),
                             act_quant_block, _stream(stream)))
    return outputs


def gemv_fp8_e4m3_ue8m0_rows(ctx, weight, scale, input, row_start, row_end, output=None,
                             act_quant_block=0, stream=None):
    out = gemv_fp8_e4m3_ue8m0_rows_multi(ctx, weight, scale, input.view(1, -1), row_start,
                                         row_end, None if output is None else output.view(1, -1),
                                         act_quant_block, stream)
    return out.view(-1)


def gemv_fp8_e4m3_ue8m0_tensorwise(ctx, weight, scale, input, output=None, act_quant_block=0,
                                   stream=None):
    return gemv_fp8_e4m3_ue8m0_rows(ctx, weight, scale, input, 0, weight.shape[0], output,
                                    act_quant_block, stream)


def fp8_act_quant_dequant_in_place(ctx, values, block_size: int = 64, stream=None):
    _check(lib().wh_act_quant_fp8(ctx.handle, _ptr(values), values.numel(), block_size,
                                  _stream(stream)))
    return values


# --------------------------------------------------------------------------
# FP4 (src/deepseek_v4.rs:410-601)
# --------------------------------------------------------------------------
@dataclass
class Fp4Matvec:
    """Fp4Matvec: packed_weight (uint8 [rows, (cols+1)//2]) and ue8m0_scales
    (uint8 [rows, scale_cols]) are CUDA tensors."""
    packed_weight: object
    ue8m0_scales: object
    rows: int
    cols: int
    scale_cols: int

    def spec(self) -> Fp4MatvecSpec:
        return Fp4MatvecSpec(_ptr(self.packed_weight), self.packed_weight.numel(),
                             _ptr(self.ue8m0_scales), self.ue8m0_scales.numel(), self.rows,
                             self.cols, self.scale_cols)


@dataclass
class DeepSeekV4Fp4Expert:
    w1: Fp4Matvec
    w3: Fp4Matvec
    w2: Fp4Matvec

    def spec(self) -> Fp4ExpertSpec:
        return Fp4ExpertSpec(self.w1.spec(), self.w3.spec(), self.w2.spec())


def fp4_e2m1_ue8m0_matvec(ctx, spec: Fp4Matvec, input, output, stream=None):
    s = spec.spec()
    _check(lib().wh_fp4_matvec(ctx.handle, C.byref(s), _ptr(input), input.numel(), _ptr(output),
                               output.numel(), _stream(stream)))
    return output


def deepseek_v4_fp4_expert_scratch_len(intermediate: int) -> int:
    return int(lib().wh_fp4_expert_scratch_len(intermediate))


def deepseek_v4_fp4_expert_forward(ctx, expert: DeepSeekV4Fp4Expert, input, output, scratch,
                                   stream=None):
    s = expert.spec()
    _check(lib().wh_fp4_expert_forward(ctx.handle, C.byref(s), _ptr(input), input.numel(),
                                       _ptr(output), output.numel(), _ptr(scratch),
                                       scratch.numel(), _stream(stream)))
    return output


def deepseek_v4_fp4_expert_forward_noalloc(ctx, expert: DeepSeekV4Fp4Expert, input, output,
                                           stream=None):
    """The expert forward with library-owned static scratch (no allocation)."""
    s = expert.spec()
    _check(lib().wh_fp4_expert_forward_noalloc(ctx.handle, C.byref(s), _ptr(input),
                                               input.numel(), _ptr(output), output.numel(),
                                               _stream(stream)))
    return output


# --------------------------------------------------------------------------
# Router (src/compute.rs:2129-2268, src/server/generation.rs:3137-3180)
# --------------------------------------------------------------------------
def route_experts(ctx, gate_bf16, x, topk: int, mode: int = ROUTER_RAW_LOGITS, bias=None,
                  route_scale: float = 1.0, hash_ids=None, logits=None, stream=None):
    """gate_bf16: int16/uint16 bits or torch.bfloat16 [experts, hidden]; x [tokens, hidden]."""
    import torch

    if x.dim() == 1:
        x = x.view(1, -1)
    E, H = gate_bf16.shape
    T = x.shape[0]
    ids = torch.empty(T, topk, dtype=torch.int32, device=x.device)
    w = torch.empty(T, topk, dtype=torch.float32, device=x.device)
    _check(lib().wh_router_topk(ctx.handle, _ptr(gate_bf16), E, H, _ptr(x), T, topk, mode,
                                _ptr(bias), route_scale, _ptr(hash_ids), _ptr(ids), _ptr(w),
                                _ptr(logits), _stream(stream)))
    return ids, w


# --------------------------------------------------------------------------
# MoE layer
# --------------------------------------------------------------------------
@dataclass
class Fp8Matrix:
    """An FP8 E4M3 matrix with UE8M0 block scales: weight uint8 [rows, cols] and
    scale uint8 [scale_rows, scale_cols] CUDA tensors."""
    weight: object
    scale: object

    def spec(self) -> Fp8MatrixSpec:
        r, c = self.weight.shape
        sr, sc = self.scale.shape
        return Fp8MatrixSpec(_ptr(self.weight), _ptr(self.scale), r, c, sr, sc)


@dataclass
class DeepSeekV4Fp8Expert:
    """DeepSeek-V4's FP8 shared expert (w1, w3 [inter, hidden], w2 [hidden, inter])."""
    w1: Fp8Matrix
    w3: Fp8Matrix
    w2: Fp8Matrix

    def spec(self) -> Fp8ExpertSpec:
        return Fp8ExpertSpec(self.w1.spec(), self.w3.spec(), self.w2.spec())


def deepseek_v4_fp8_expert_forward(ctx, expert: DeepSeekV4Fp8Expert, input, output, scratch,
                                   stream=None):
    """compute_deepseek_fp8_shared_expert_into_hidden (src/compute.rs:5545-5614)."""
    s = expert.spec()
    _check(lib().wh_fp8_expert_forward(ctx.handle, C.byref(s), _ptr(input), input.numel(),
                                       _ptr(output), output.numel(), _ptr(scratch),
                                       scratch.numel(), _stream(stream)))
    return output


def lm_head_topk_score(ctx: Context, weight_bf16, x, top_k: int, row_base: int = 0,
                       logits=None, scratch=None, stream=None):
    """score_bf16_lm_head_topk + push_topk_candidate + the final sort
    (src/compute.rs:2838-2962) on the device: weight_bf16 [rows, cols] (bf16 bits as
    int16/uint16, or a bfloat16 tensor), x [cols] f32.  Returns (tokens int32,
    logits f32) of min(top_k, rows) entries, sorted descending."""
    import torch

    rows, cols = weight_bf16.shape
    k = max(int(top_k), 1)
    n = min(k, rows)
    dev = weight_bf16.device
    toks = torch.empty(max(k, 1), dtype=torch.int32, device=dev)
    vals = torch.empty(max(k, 1), dtype=torch.float32, device=dev)
    if scratch is None:
        scratch = torch.empty(lib().wh_lm_head_scratch_bytes(rows, k), dtype=torch.uint8,
                              device=dev)
    _check(lib().wh_lm_head_topk(ctx.handle, _ptr(weight_bf16), rows, cols, row_base, _ptr(x),
                                 x.numel(), k, _ptr(toks), _ptr(vals), _ptr(logits),
                                 _ptr(scratch), scratch.numel(), _stream(stream)))
    return toks[:n], vals[:n]


def lm_head_topk_score_batch(ctx: Context, weight_bf16, x, top_k: int, row_base: int = 0,
                             logits=None, scratch=None, stream=None):
    """lm_head_topk_score for every row of x [tokens, cols] at once (the
    weight streams once per tile of up to 8 tokens).  Returns (tokens int32
    [T, min(top_k, rows)], logits f32 [T, min(top_k, rows)]); row t equals
    lm_head_topk_score(x[t]) bit for bit."""
    import torch

    rows, cols = weight_bf16.shape
    T = x.shape[0]
    k = max(int(top_k), 1)
    n = min(k, rows)
    dev = weight_bf16.device
    toks = torch.empty(T, k, dtype=torch.int32, device=dev)
    vals = torch.empty(T, k, dtype=torch.float32, device=dev)
    if scratch is None:
        scratch = torch.empty(lib().wh_lm_head_batch_scratch_bytes(rows, k, T),
                              dtype=torch.uint8, device=dev)
    _check(lib().wh_lm_head_topk_batch(ctx.handle, _ptr(weight_bf16), rows, cols, row_base,
                                       _ptr(x), T, x.stride(0), k, _ptr(toks), _ptr(vals),
                                       _ptr(logits), _ptr(scratch), scratch.numel(),
                                       _stream(stream)))
    return toks[:, :n], vals[:, :n]


# DeepSeek-V4's attention constants (src/compute.rs DEEPSEEK_V4_YARN,
# DEEPSEEK_V4_COMPRESS_ROPE_THETA, DEEPSEEK_V4_SLIDING_WINDOW_SIZE)
DEEPSEEK_V4_YARN = (16.0, 32.0, 1.0, 65536)
DEEPSEEK_V4_COMPRESS_ROPE_THETA = 160000.0
DEEPSEEK_V4_ROPE_THETA = 10000.0
DEEPSEEK_V4_SLIDING_WINDOW = 128
# DEEPSEEK_V4_COMPRESS_RATIOS (src/compute.rs:2551-2554): per physical layer
DEEPSEEK_V4_COMPRESS_RATIOS = (0, 0) + (4, 128) * 20 + (4, 0)


def deepseek_rope_for_layer(layer: int):
    """deepseek_rope_for_layer (src/compute.rs:2575-2585): (theta, yarn or None)."""
    ratio = DEEPSEEK_V4_COMPRESS_RATIOS[layer] if 0 <= layer < len(DEEPSEEK_V4_COMPRESS_RATIOS) else 0
    if ratio > 0:
        return DEEPSEEK_V4_COMPRESS_ROPE_THETA, DEEPSEEK_V4_YARN
    return DEEPSEEK_V4_ROPE_THETA, None


def rope_inv_freqs(rope_dim: int, theta: float, yarn=None):
    """rope_inv_freqs (src/compute.rs:2591-2621): per-pair inverse frequencies,
    YaRN-blended when yarn = (factor, beta_fast, beta_slow, original_seq_len)."""
    import numpy as np

    out = np.zeros(rope_dim // 2, np.float32)
    fa, bf, bs, osl = yarn if yarn else (0.0, 0.0, 0.0, 0)
    lib().wh_rope_inv_freqs(rope_dim, theta, fa, bf, bs, osl, out.ctypes.data)
    return out


def mla_attention(ctx: Context, q, keys, token_pos: int, inv_freqs, nope_dim: int,
                  window: int = DEEPSEEK_V4_SLIDING_WINDOW, compressed=None, sink=None,
                  out=None, stream=None):
    """The attention core of compute_deepseek_v4_mla_attention
    (src/compute.rs:4080-4185) on the device, bit-exact: q [heads, head_dim] f32,
    keys [positions > token_pos, key_stride] f32 (the layer's latent KV cache rows;
    key and value are the same row), compressed [count, head_dim] f32 or None,
    sink [heads] f32 or None, inv_freqs: the layer's rope_inv_freqs (host array).
    Returns out [heads, head_dim]."""
    import numpy as np
    import torch

    heads, head_dim = q.shape
    if out is None:
        out = torch.empty(heads, head_dim, dtype=torch.float32, device=q.device)
    fr = np.ascontiguousarray(inv_freqs, dtype=np.float32)
    cc = 0 if compressed is None else compressed.shape[0]
    _check(lib().wh_mla_attention(ctx.handle, _ptr(q), heads, head_dim, nope_dim, _ptr(keys),
                                  keys.stride(0), token_pos, window, _ptr(compressed), cc,
                                  _ptr(sink), fr.ctypes.data if fr.size else None, _ptr(out),
                                  _stream(stream)))
    return out


# DeepSeek-V4's hyper-connection settings (src/compute.rs ComputeConfig)
DEEPSEEK_V4_HC_MULT = 4
DEEPSEEK_V4_HC_SINKHORN_ITERS = 20
DEEPSEEK_V4_HC_EPS = 1.0e-6


def hc_pre(ctx: Context, fn, scale, base, x, hc: int, hidden: int,
           sinkhorn_iters: int = DEEPSEEK_V4_HC_SINKHORN_ITERS,
           eps: float = DEEPSEEK_V4_HC_EPS, out=None, stream=None):
    """hc_pre_into + hc_split_sinkhorn_scalar (src/compute.rs:4945-5053) on the
    device for x [tokens, hc * hidden] f32: returns (y [tokens, hidden],
    post [tokens, hc], comb [tokens, hc, hc]).  fn [(2 + hc) * hc, hc * hidden],
    scale [3] and base [(2 + hc) * hc] are f32 device tensors."""
    import torch

    tokens = x.shape[0]
    dev = x.device
    if out is None:
        out = (torch.empty(tokens, hidden, device=dev), torch.empty(tokens, hc, device=dev),
               torch.empty(tokens, hc, hc, device=dev))
    y, post, comb = out
    _check(lib().wh_hc_pre(ctx.handle, _ptr(fn), _ptr(scale), _ptr(base), _ptr(x), tokens, hc,
                           hidden, sinkhorn_iters, eps, _ptr(y), _ptr(post), _ptr(comb),
                           _stream(stream)))
    return y, post, comb


def hc_post(ctx: Context, y, residual, post, comb, hc: int, hidden: int, out=None,
            stream=None):
    """hc_post_into (src/compute.rs:5055-5089): out [tokens, hc * hidden]."""
    import torch

    tokens = y.shape[0]
    if out is None:
        out = torch.empty(tokens, hc * hidden, device=y.device)
    _check(lib().wh_hc_post(ctx.handle, _ptr(y), _ptr(residual), _ptr(post), _ptr(comb),
                            tokens, hc, hidden, _ptr(out), _stream(stream)))
    return out


def hc_head(ctx: Context, fn, scale: float, base, x, hc: int, hidden: int,
            eps: float = DEEPSEEK_V4_HC_EPS, out=None, stream=None):
    """hc_head_pool (src/compute.rs:5091-5132): pooled [tokens, hidden]."""
    import torch

    tokens = x.shape[0]
    if out is None:
        out = torch.empty(tokens, hidden, device=x.device)
    _check(lib().wh_hc_head(ctx.handle, _ptr(fn), float(scale), _ptr(base), _ptr(x), tokens,
                            hc, hidden, eps, _ptr(out), _stream(stream)))
    return out


# --------------------------------------------------------------------------
# DeepSeek-V4 attention block (src/compute.rs:3077-3115, 3924-4293)
# --------------------------------------------------------------------------
def rms_norm(ctx: Context, x, weight_bf16=None, out=None, stream=None):
    """apply_weighted_rms_norm (weight: bf16 bits [n]) or rms_norm_in_place
    (weight None) of every row of x [..., n] f32 on the device."""
    import torch

    n = x.shape[-1]
    if out is None:
        out = torch.empty_like(x)
    _check(lib().wh_rms_norm(ctx.handle, _ptr(x), _ptr(out), x.numel() // n, n,
                             _ptr(weight_bf16), _stream(stream)))
    return out


def gemv_fp8_e4m3_ue8m0_grouped(ctx: Context, weight, scale, x, group_rows: int,
                                group_offset: int, row_start: int = 0, row_end=None, out=None,
                                act_quant_block: int = 0, stream=None):
    """The reference's grouped wo_a (gemv_fp8_e4m3_ue8m0_rows per group): row r
    reads x[(r // group_rows) * group_offset:][:cols]."""
    import torch

    rows, cols = weight.shape
    srows, scols = scale.shape
    row_end = rows if row_end is None else row_end
    if out is None:
        out = torch.empty(row_end - row_start, device=x.device, dtype=torch.float32)
    _check(lib().wh_fp8_gemv_grouped(ctx.handle, _ptr(weight), _ptr(scale), rows, cols, srows,
                                     scols, row_start, row_end, _ptr(x), 1, x.numel(),
                                     group_rows, group_offset, _ptr(out), out.numel(),
                                     act_quant_block, _stream(stream)))
    return out


class V4AttnSpec(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "heads", "head_dim", "nope_dim", "q_lora_rank",
                                       "o_groups", "o_lora_rank", "window")] + [
        ("wq_a", Fp8MatrixSpec), ("wq_b", Fp8MatrixSpec), ("wkv", Fp8MatrixSpec),
        ("wo_a", Fp8MatrixSpec), ("wo_b", Fp8MatrixSpec), ("q_norm", C.c_void_p),
        ("kv_norm", C.c_void_p), ("sink", C.c_void_p)]


@dataclass
class V4Attention:
    """One layer's MLA attention weights (device tensors): Fp8Matrix projections,
    bf16-bit norms (or None) and the attention sink (or None)."""
    wq_a: "Fp8Matrix"
    wq_b: "Fp8Matrix"
    wkv: "Fp8Matrix"
    wo_a: "Fp8Matrix"
    wo_b: "Fp8Matrix"
    q_norm: object = None
    kv_norm: object = None
    sink: object = None
    hidden: int = 4096
    heads: int = 64
    head_dim: int = 512
    nope_dim: int = 448
    q_lora_rank: int = 1024
    o_groups: int = 8
    o_lora_rank: int = 1024
    window: int = DEEPSEEK_V4_SLIDING_WINDOW

    def spec(self) -> V4AttnSpec:
        return V4AttnSpec(self.hidden, self.heads, self.head_dim, self.nope_dim,
                          self.q_lora_rank, self.o_groups, self.o_lora_rank, self.window,
                          self.wq_a.spec(), self.wq_b.spec(), self.wkv.spec(), self.wo_a.spec(),
                          self.wo_b.spec(), _ptr(self.q_norm), _ptr(self.kv_norm),
                          _ptr(self.sink))


def v4_attention_scratch_len(layer: V4Attention, tokens: int = 1) -> int:
    s = layer.spec()
    return int(lib().wh_v4_attention_scratch_len(C.byref(s), tokens))


def v4_attention(ctx: Context, layer: V4Attention, token_pos, hidden, kv_caches, inv_freqs,
                 compressed=None, scratch=None, stream=None):
    """compute_deepseek_v4_mla_attention on the device, bit-exact, for one
    token (token_pos an int, hidden [hidden], kv_caches one [positions, stride]
    tensor, compressed one tensor or None) or for a batch (token_pos a list,
    hidden [tokens, hidden], kv_caches / compressed lists, one per token).
    hidden is overwritten by the attention outputs; each token's KV cache gets
    its row token_pos."""
    import numpy as np
    import torch

    single = isinstance(token_pos, int)
    pos = [token_pos] if single else list(token_pos)
    kvs = [kv_caches] if single else list(kv_caches)
    comps = [compressed] if single else list(compressed or [None] * len(pos))
    T = len(pos)
    s = layer.spec()
    n = int(lib().wh_v4_attention_scratch_len(C.byref(s), T))
    if scratch is None or scratch.numel() < n:
        scratch = torch.empty(n, dtype=torch.float32, device=hidden.device)
    fr = np.ascontiguousarray(inv_freqs, dtype=np.float32)
    pos_a = (C.c_int * T)(*pos)
    kv_a = (C.c_void_p * T)(*[_ptr(k) for k in kvs])
    cp_a = (C.c_void_p * T)(*[_ptr(c) for c in comps])
    cc_a = (C.c_int * T)(*[0 if c is None else c.shape[0] for c in comps])
    _check(lib().wh_v4_attention(ctx.handle, C.byref(s), T, pos_a, _ptr(hidden), kv_a,
                                 kvs[0].stride(0), cp_a, cc_a,
                                 fr.ctypes.data if fr.size else None, _ptr(scratch),
                                 scratch.numel(), _stream(stream)))
    return hidden


class MoeLayer:
    """A prepared MoE FFN layer (router + routed FP4 experts + shared expert).

    forward(x) replaces routing + compute_active_and_shared_experts
    (src/compute.rs:1872-2030) for each token of x [tokens, hidden].
    """

    def __init__(self, ctx: Context, experts: Sequence[DeepSeekV4Fp4Expert],
                 shared, gate_bf16, topk: int = 6,
                 router_mode: int = ROUTER_RAW_LOGITS, route_scale: float = 1.0,
                 gate_bias=None, max_tokens: int = 1, exact: int = 0):
        """shared: a DeepSeekV4Fp4Expert, a DeepSeekV4Fp8Expert (DeepSeek-V4's
        layout) or None."""
        import torch

        self.ctx = ctx
        self.hidden = experts[0].w1.cols
        self.inter = experts[0].w1.rows
        self.topk = topk
        self._experts = list(experts)
        self._shared = shared
        self._gate = gate_bf16
        self._bias = gate_bias
        arr = (Fp4ExpertSpec * len(experts))(*[e.spec() for e in experts])
        fp8 = isinstance(shared, DeepSeekV4Fp8Expert)
        sh = shared.spec() if shared is not None else None
        d = MoeDesc(len(experts), self.hidden, self.inter, arr,
                    C.pointer(sh) if sh is not None and not fp8 else None, _ptr(gate_bf16),
                    _ptr(gate_bias), topk, router_mode, route_scale, max_tokens, int(exact),
                    C.pointer(sh) if fp8 else None)
        h = C.c_void_p()
        _check(lib().wh_moe_plan_create(ctx.handle, C.byref(d), C.byref(h)))
        self.plan = h
        self.max_tokens = max_tokens
        # the per-token path (fewer than 32 tokens) and the grouped path lay
        # scratch out differently: size for the larger of the two
        nbytes = max(lib().wh_moe_scratch_bytes(h, t) for t in {max_tokens, min(max_tokens, 31)})
        self.scratch = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{ctx.device}")

    def forward(self, x, y=None, ids=None, weights=None, hash_ids=None, stream=None):
        import torch

        if x.dim() == 1:
            x = x.view(1, -1)
        T = x.shape[0]
        if y is None:
            y = torch.empty_like(x)
        _check(lib().wh_moe_ffn(self.ctx.handle, self.plan, _ptr(x), T, _ptr(hash_ids), _ptr(y),
                                _ptr(ids), _ptr(weights), _ptr(self.scratch), self.scratch.numel(),
                                _stream(stream)))
        return y

    def scratch_field(self, tokens: int, field: int, dtype, shape):
        """A view of one intermediate array of the last grouped (tensor-core)
        call of `tokens` tokens (MOE_FIELD_*), read from the layer's scratch."""
        import torch

        off, n = C.c_size_t(), C.c_size_t()
        _check(lib().wh_moe_scratch_field(self.plan, tokens, field, C.byref(off), C.byref(n)))
        es = torch.empty((), dtype=dtype).element_size()
        count = 1
        for d in shape:
            count *= d
        if count * es > n.value:
            raise ValueError(f"field {field}: {count * es} bytes asked, {n.value} there")
        return self.scratch[off.value:off.value + count * es].view(dtype).view(*shape)

    def set_fused_decode(self, on: bool = True) -> None:
        """One-token calls as one persistent kernel (on) or as three kernels (default)."""
        _check(lib().wh_moe_plan_set_fused_decode(self.plan, 1 if on else 0))

    def close(self):
        if getattr(self, "plan", None):
            lib().wh_moe_plan_destroy(self.plan)
            self.plan = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
