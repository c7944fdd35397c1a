"""Python view of libk3gpu.so, the B200 speculative-verification library.

This mirrors the C ABI of ``include/k3gpu.h`` one function at a time (ctypes, device
pointers taken from torch CUDA tensors). torch is only the plumbing here -- device
memory and streams; every computation runs in the library's own sm_100a kernels. There
is no CPU fallback: importing this module on a box without the built library, or calling
it without a CUDA device, raises.

The directory name is not a Python identifier, so callers load it by path::

    spec = importlib.util.spec_from_file_location("k3b200", "<repo>/kimi-k3-for-me_b200/__init__.py")
"""
from __future__ import annotations

import ctypes as C
import os

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libk3gpu.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python {os.path.join(PKG, 'build.py')}` "
        "(there is no CPU fallback for this library)")

lib = C.CDLL(LIB_PATH)

VP, I, F, SZ = C.c_void_p, C.c_int, C.c_float, C.c_size_t
U64 = C.c_uint64

K3GPU_OK, K3GPU_EINVAL, K3GPU_ECAPACITY, K3GPU_ECUDA, K3GPU_EDEVICE = 0, -1, -2, -3, -4
ACT_SITU, ACT_SWIGLU = 0, 1


class K3GpuExpertBank(C.Structure):
    _fields_ = [("base", VP), ("stride", C.c_int64), ("p1", C.c_int64), ("s1", C.c_int64),
                ("p2", C.c_int64), ("s2", C.c_int64), ("p3", C.c_int64), ("s3", C.c_int64),
                ("n_experts", I), ("L", I), ("I", I), ("f16_safe", VP), ("n_f16_unsafe", I)]


class K3GpuLayerCfg(C.Structure):
    _fields_ = [("hidden", I), ("kda_heads", I), ("kda_head_dim", I), ("conv_k", I), ("gate_lb", F),
                ("rms_eps", F), ("attn_res_block", I), ("max_blocks", I), ("n_routed", I), ("n_shared", I),
                ("topk", I), ("moe_inter", I), ("act", I), ("renorm", I), ("routed_scale", F), ("situ_b1", F),
                ("situ_b2", F), ("latent", I), ("shared_inter", I), ("mla_heads", I), ("q_lora", I),
                ("kv_lora", I), ("qk_nope", I), ("qk_rope", I), ("v_head", I)]


class K3GpuMoeCfg(C.Structure):
    _fields_ = [("hidden", I), ("latent", I), ("moe_inter", I), ("shared_inter", I), ("n_routed", I), ("topk", I),
                ("act", I), ("renorm", I), ("routed_scale", F), ("situ_b1", F), ("situ_b2", F), ("rms_eps", F)]


class K3GpuMoeW(C.Structure):
    _fields_ = [(n, VP) for n in ("down", "up", "sh1", "sh3", "sh2", "gate_W", "gate_bias", "latent_norm")] + \
               [("bank", C.POINTER(K3GpuExpertBank))]


class K3GpuKdaW(C.Structure):
    _fields_ = [(n, VP) for n in ("q", "k", "v", "b", "f_a", "f_b", "g", "o", "q_conv", "k_conv", "v_conv",
                                  "A_log", "dt_bias", "o_norm")]


class K3GpuKdaLog(C.Structure):
    _fields_ = [(n, VP) for n in ("k", "v", "alpha", "beta", "pre")]


class K3GpuKdaLayerW(C.Structure):
    _fields_ = [("attn_res_fold", VP), ("mlp_res_fold", VP), ("in_norm", VP), ("post_norm", VP),
                ("kda", K3GpuKdaW), ("gate_W", VP), ("gate_bias", VP), ("bank", C.POINTER(K3GpuExpertBank)),
                ("moe", C.POINTER(K3GpuMoeW))]


class K3GpuMlaW(C.Structure):
    _fields_ = [(n, VP) for n in ("q_a", "q_b", "kv_a", "g", "o", "q_a_norm", "kv_a_norm", "kv_b")]


class K3GpuMlaLayerW(C.Structure):
    _fields_ = [("attn_res_fold", VP), ("mlp_res_fold", VP), ("in_norm", VP), ("post_norm", VP),
                ("mla", K3GpuMlaW), ("gate_W", VP), ("gate_bias", VP), ("bank", C.POINTER(K3GpuExpertBank)),
                ("moe", C.POINTER(K3GpuMoeW))]


class K3GpuModelCfg(C.Structure):
    _fields_ = [("layer", K3GpuLayerCfg), ("n_layers", I), ("vocab", I), ("is_mla", VP)]


class K3GpuModelW(C.Structure):
    _fields_ = [("embed", VP), ("lm_head", VP), ("norm", VP), ("out_res_fold", VP),
                ("kda", C.POINTER(K3GpuKdaLayerW)), ("mla", C.POINTER(K3GpuMlaLayerW))]


EP_MAX_WORLD = 8
EP_HANDLE_BYTES = 64


class K3StateLayout(C.Structure):
    _fields_ = [("fp", I * 12), ("n_bound", I), ("n_mla", I), ("kper", C.c_int64), ("kvpp", C.c_int64),
                ("ropepp", C.c_int64), ("loop_a", I), ("loop_b", I), ("loop_count", I), ("loop_nv", I),
                ("loop_eps", C.c_double)]


class K3SpecCost(C.Structure):
    """The drafting study's verify-step cost model (units of one plain decode step)."""
    _fields_ = [("a_T", C.c_double), ("a_E", C.c_double), ("a_C", C.c_double), ("eps", C.c_double),
                ("expert_ratio", C.c_double)]


SPEC_P3_CODES = 234

DRAFT_NONE, DRAFT_NGRAM, DRAFT_EAGER, DRAFT_SUFFIX, DRAFT_P3, DRAFT_TREE, DRAFT_MODEL = range(7)
SPEC_LOOP_GEN, SPEC_LOOP_STOP_ID, SPEC_LOOP_CONTEXT, SPEC_LOOP_PAUSED = 1, 2, 3, 4


class K3SpecLoopCfg(C.Structure):
    _fields_ = [("policy", I), ("spec_n", I), ("min_len", I), ("gen", I), ("tmax", I), ("kv_cap", I),
                ("stop_ids", VP), ("n_stop", I), ("p3_q", VP), ("p3_delta", C.c_double), ("p3_cost", VP),
                ("p3_replay", I), ("tree_nodes", I), ("tree_branch", I), ("prefill_chunk", I), ("pause_after", I)]


class K3SpecLoopStats(C.Structure):
    _fields_ = [(n, C.c_longlong) for n in ("steps", "sweeps", "drafted", "accepted", "dropped", "full",
                                            "partial", "cut")] + [("hist", C.c_longlong * 9)] + \
               [(n, C.c_longlong) for n in ("draft_rounds", "draft_drafted", "draft_accepted", "draft_dropped")]


class K3SpecStepTrace(C.Structure):
    _fields_ = [("nd", I), ("m", I), ("keep", I), ("fed", I)]


SpecVerifyFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int, C.c_int,
                           C.POINTER(C.c_int))
SpecCommitFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_int), C.c_int)
SpecCheckpointFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int)


ST_UNKNOWN, ST_U8, ST_BF16, ST_F16, ST_F32 = range(5)


class K3StTensorInfo(C.Structure):
    _fields_ = [("dtype", I), ("dtype_name", C.c_char * 16), ("ndim", I), ("shape", C.c_int64 * 8),
                ("shard", I), ("nbytes", C.c_int64)]


class K3GpuEpGroup(C.Structure):
    _fields_ = [("arena", VP * EP_MAX_WORLD), ("world", I), ("rank", I), ("cap", I), ("L", I), ("K", I),
                ("n_local", I)]


_SIGS = {
    "k3gpu_strerror": ([I], C.c_char_p),
    "k3gpu_last_cuda_error": ([], I),
    "k3gpu_version": ([], I),
    "k3gpu_launch_count": ([], C.c_longlong),
    "k3gpu_model_last_routing": ([VP, C.POINTER(VP)], I),
    "k3gpu_device_status": ([I, C.POINTER(I)], I),
    "k3gpu_router_workspace": ([I, I], SZ),
    "k3gpu_router": ([VP, VP, VP, VP, VP, I, I, I, I, I, F, VP, SZ, VP], I),
    "k3gpu_router_noalloc": ([VP, VP, VP, VP, VP, I, I, I, I, I, F, VP], I),
    "k3gpu_bank_layout": ([C.POINTER(K3GpuExpertBank), I, I], None),
    "k3gpu_mxfp4_dequant": ([VP, VP, VP, I, I, VP], I),
    "k3gpu_bank_scan": ([C.POINTER(K3GpuExpertBank), VP, VP], I),
    "k3gpu_moe_workspace": ([I, I, I, I, I, I], SZ),
    "k3gpu_moe_experts": ([VP, VP, VP, VP, C.POINTER(K3GpuExpertBank), I, I, I, I, I, F, F, VP,
                           F, VP, SZ, VP], I),
    "k3gpu_moe_layer": ([VP, VP, VP, VP, VP, VP, C.POINTER(K3GpuExpertBank), I, I, I, I, I, F, F,
                         I, F, VP, SZ, VP], I),
    "k3gpu_moe_select_kernels": ([I], I),
    "k3gpu_moe_phase_timing": ([I], I),
    "k3gpu_moe_phase_ms": ([C.POINTER(F), I], I),
    "k3gpu_kda_verify": ([VP, VP, VP, VP, VP, VP, VP, I, I, I, I, F, VP], I),
    "k3gpu_kda_verify_tree": ([VP] * 8 + [I, I, I, I, F, VP], I),
    "k3gpu_kda_prologue_tree": ([VP] * 15 + [I, I, I, I, I, F, VP], I),
    "k3gpu_kda_commit": ([VP, VP, VP, VP, VP, VP, I, I, I, I, VP], I),
    "k3gpu_kda_prefill": ([VP] * 7 + [I, I, I, I, F, VP], I),
    "k3gpu_kda_prologue": ([VP] * 14 + [I, I, I, I, I, F, VP], I),
    "k3gpu_kda_commit_conv": ([VP, VP, VP, I, I, I, I, I, VP], I),
    "k3gpu_kda_norm_gate": ([VP, VP, VP, I, I, I, F, VP], I),
    "k3gpu_mla_workspace": ([I, I, I, I, I], SZ),
    "k3gpu_mla_absorbed": ([VP] * 8 + [I] * 9 + [F, VP, SZ, VP], I),
    "k3gpu_argmax": ([VP, VP, I, I, VP], I),
    "k3gpu_model_arena_bytes": ([C.POINTER(K3GpuModelCfg), I, I, I], SZ),
    "k3gpu_model_create": ([C.POINTER(K3GpuModelCfg), C.POINTER(K3GpuModelW), I, I, I, VP, SZ, VP], VP),
    "k3gpu_model_free": ([VP], None),
    "k3gpu_model_set_stream": ([VP, VP], I),
    "k3gpu_model_reset": ([VP], I),
    "k3gpu_model_verify": ([VP, VP, I, VP, VP, C.POINTER(VP)], I),
    "k3gpu_model_verify_greedy": ([VP, VP, I, VP, VP], I),
    "k3gpu_model_commit": ([VP, VP, VP], I),
    "k3gpu_model_commit_device": ([VP, VP, VP], I),
    "k3gpu_model_prefill": ([VP, VP, I, VP], I),
    "k3gpu_model_cached": ([VP, VP], I),
    "k3gpu_model_set_cached": ([VP, VP], I),
    "k3gpu_model_kda_state": ([VP, I, C.POINTER(VP), C.POINTER(VP)], I),
    "k3gpu_model_mla_cache": ([VP, I, C.POINTER(VP), C.POINTER(VP)], I),
    "k3gpu_model_loop_verify": ([VP, VP, VP, I, I, VP], I),
    "k3gpu_model_loop_commit": ([VP, I, VP, I], I),
    "k3gpu_accept_greedy": ([VP, VP, VP, VP, VP, VP, I, I, I, VP], I),
    "k3gpu_accept_tree_greedy": ([VP] * 7 + [I, I, I, VP], I),
    "k3gpu_accept_sample": ([VP] * 5 + [I, I, I, F, U64, U64, VP], I),
    "k3gpu_rmsnorm": ([VP, VP, VP, I, I, F, VP], I),
    "k3gpu_matmul_bf16_workspace": ([I, I, I], SZ),
    "k3gpu_matmul_bf16_batch": ([VP, I, VP, I, VP, I, I, I, VP, SZ, VP], I),
    "k3gpu_lm_head_argmax_workspace": ([I, I, I], SZ),
    "k3gpu_lm_head_argmax": ([VP, VP, I, VP, I, I, I, VP, SZ, VP], I),
    "k3gpu_attn_res": ([VP, VP, VP, VP, VP, I, I, I, F, VP], I),
    "k3gpu_moe_prefill_workspace": ([C.POINTER(K3GpuMoeCfg), I], SZ),
    "k3gpu_moe_prefill": ([VP, VP, VP, VP, C.POINTER(K3GpuMoeW), C.POINTER(K3GpuMoeCfg), I, VP, SZ, VP], I),
    "k3gpu_kda_layer_workspace": ([C.POINTER(K3GpuLayerCfg), I, I], SZ),
    "k3gpu_kda_layer_verify": ([VP, VP, C.POINTER(K3GpuKdaW), C.POINTER(K3GpuLayerCfg), VP, VP,
                                C.POINTER(K3GpuKdaLog), I, I, VP, SZ, VP], I),
    "k3gpu_decoder_layer_workspace": ([C.POINTER(K3GpuLayerCfg), I, I], SZ),
    "k3gpu_decoder_layer_kda_verify": ([VP, VP, VP, VP, VP, C.POINTER(K3GpuKdaLayerW), C.POINTER(K3GpuLayerCfg), I,
                                        VP, VP, C.POINTER(K3GpuKdaLog), I, I, VP, SZ, VP], I),
    "k3gpu_mla_layer_workspace": ([C.POINTER(K3GpuLayerCfg), I, I, I], SZ),
    "k3gpu_mla_layer_verify": ([VP, VP, C.POINTER(K3GpuMlaW), C.POINTER(K3GpuLayerCfg), VP, VP, I, VP, VP, I, I, I,
                                VP, SZ, VP], I),
    "k3gpu_decoder_layer_mla_workspace": ([C.POINTER(K3GpuLayerCfg), I, I, I], SZ),
    "k3gpu_decoder_layer_mla_verify": ([VP, VP, VP, VP, VP, C.POINTER(K3GpuMlaLayerW), C.POINTER(K3GpuLayerCfg), I,
                                        VP, VP, I, VP, VP, I, I, I, VP, SZ, VP], I),
    "k3gpu_ep_arena_bytes": ([I, I, I, I], SZ),
    "k3gpu_ep_arena_alloc": ([C.POINTER(VP), SZ], I),
    "k3gpu_ep_arena_free": ([VP], I),
    "k3gpu_ep_ipc_handle": ([VP, VP], I),
    "k3gpu_ep_ipc_open": ([VP, C.POINTER(VP)], I),
    "k3gpu_ep_ipc_close": ([VP], I),
    "k3gpu_ep_recv_views": ([C.POINTER(K3GpuEpGroup), C.POINTER(VP), C.POINTER(VP), C.POINTER(VP)], I),
    "k3gpu_ep_dispatch": ([C.POINTER(K3GpuEpGroup), VP, VP, VP, I, C.c_uint, VP, VP], I),
    "k3gpu_ep_receive": ([C.POINTER(K3GpuEpGroup), C.c_uint, VP], I),
    "k3gpu_ep_return": ([C.POINTER(K3GpuEpGroup), VP, C.c_uint, VP], I),
    "k3gpu_ep_combine": ([C.POINTER(K3GpuEpGroup), VP, VP, I, C.c_uint, VP, VP], I),
    "k3gpu_ep_set_wait_limit": ([C.c_longlong], I),
    "k3gpu_moe_layer_ep_workspace": ([C.POINTER(K3GpuEpGroup), I, I, I, I], SZ),
    "k3gpu_moe_layer_ep": ([VP, VP, VP, VP, VP, VP, C.POINTER(K3GpuExpertBank), C.POINTER(K3GpuExpertBank),
                            C.POINTER(K3GpuEpGroup), C.c_uint, I, I, I, I, I, F, F, I, F, VP, VP, SZ, VP], I),
    "k3gpu_model_ep_workspace": ([VP, C.POINTER(K3GpuEpGroup)], SZ),
    "k3gpu_model_set_ep": ([VP, C.POINTER(K3GpuEpGroup), VP, VP, SZ], I),
    "k3gpu_model_ep_status": ([VP, VP], I),
    "k3_spec_draft_ngram": ([VP, I, I, I, I, VP], I),
    "k3_spec_draft_eager": ([VP, I, I, VP], I),
    "k3_bank_read_safetensors": ([C.POINTER(C.c_char_p), I, I, I, I, I, I, VP, SZ], I),
    "k3_state_save": ([C.c_char_p, C.POINTER(K3StateLayout), VP, I, I, VP, VP, VP, I, VP, VP], I),
    "k3_state_peek": ([C.c_char_p, C.POINTER(K3StateLayout), C.POINTER(I), C.POINTER(I)], I),
    "k3_state_load": ([C.c_char_p, C.POINTER(K3StateLayout), VP, I, VP, VP, VP, I, VP, VP, C.POINTER(I),
                       C.POINTER(I)], I),
    "k3_suffix_drafter_create": ([I], VP),
    "k3_suffix_drafter_free": ([VP], None),
    "k3_suffix_drafter_push": ([VP, VP, I], I),
    "k3_suffix_drafter_length": ([VP], I),
    "k3_suffix_drafter_draft": ([VP, I, I, VP, C.POINTER(I), C.POINTER(I)], I),
    "k3_suffix_drafter_tree": ([VP, I, I, I, I, VP, VP], I),
    "k3_spec_loop_create": ([VP, VP, I, I, VP, VP, VP], VP),
    "k3_spec_loop_free": ([VP], None),
    "k3_spec_loop_step": ([VP, VP, VP, VP], I),
    "k3_spec_loop_state": ([VP, VP, VP, VP, VP], I),
    "k3_spec_loop_ids": ([VP, VP, I], I),
    "k3_spec_loop_set_draft_model": ([VP, VP, VP, VP], I),
    "k3_spec_loop_set_checkpoint": ([VP, VP, VP], I),
    "k3_spec_loop_request_pause": ([VP], None),
    "k3_layer_loop_plan": ([I, I, I, I, I, I, VP, I, VP, VP], I),
    "k3_st_open": ([C.c_char_p], VP),
    "k3_st_open_files": ([VP, I], VP),
    "k3_st_close": ([VP], None),
    "k3_st_count": ([VP], I),
    "k3_st_name": ([VP, I], C.c_char_p),
    "k3_st_find": ([VP, C.c_char_p, VP], I),
    "k3_st_read": ([VP, C.c_char_p, VP, SZ], C.c_int64),
    "k3_suffix_drafter_features": ([VP, VP, I, VP], I),
    "k3_spec_p3_length": ([VP, I, VP, C.c_double, I], I),
    "k3_spec_p3_cost_length": ([VP, I, VP, VP, I], I),
    "k3_suffix_drafter_draft_p3": ([VP, VP, C.c_double, VP, I, I, VP], I),
}
for _name, (_args, _res) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _res


class K3Error(RuntimeError):
    pass


def check(status: int, what: str = "") -> None:
    if status != K3GPU_OK:
        msg = lib.k3gpu_strerror(status).decode()
        if status == K3GPU_ECUDA:
            msg += f" (cudaError {lib.k3gpu_last_cuda_error()})"
        raise K3Error(f"{what}: {msg} [{status}]")


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise K3Error("expected a CUDA tensor")
    if not t.is_contiguous():
        raise K3Error("expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


def stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def device_status(device: int = 0) -> int:
    v = C.c_int(0)
    check(lib.k3gpu_device_status(device, C.byref(v)), "device_status")
    return v.value


def workspace(nbytes: int, device="cuda") -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# ------------------------------------------------------------------------- router --
def router(x, W, bias, topk, renorm=1, routed_scale=1.0, ws=None, stream=None):
    T, hidden = x.shape
    n = W.shape[0]
    idx = torch.empty((T, topk), dtype=torch.int32, device=x.device)
    w = torch.empty((T, topk), dtype=torch.float32, device=x.device)
    need = lib.k3gpu_router_workspace(T, n)
    ws = ws if ws is not None else workspace(need, x.device)
    check(lib.k3gpu_router(ptr(idx), ptr(w), ptr(x), ptr(W), ptr(bias), T, hidden, n, topk,
                           renorm, float(routed_scale), ptr(ws), ws.numel(), stream_ptr(stream)),
          "k3gpu_router")
    return idx, w


# ----------------------------------------------------------------------- experts ---
def mxfp4_dequant(packed, scales, stream=None):
    rows, half = packed.shape
    out = torch.empty((rows, 2 * half), dtype=torch.float32, device=packed.device)
    check(lib.k3gpu_mxfp4_dequant(ptr(out), ptr(packed), ptr(scales), rows, 2 * half,
                                  stream_ptr(stream)), "k3gpu_mxfp4_dequant")
    return out


class ExpertBank:
    """MXFP4 experts resident in HBM in the reference's per-expert run layout."""

    def __init__(self, bank_bytes: torch.Tensor, n_experts: int, L: int, I_: int):
        self.bytes = bank_bytes
        self.desc = K3GpuExpertBank()
        lib.k3gpu_bank_layout(C.byref(self.desc), L, I_)
        self.desc.base = bank_bytes.data_ptr()
        self.desc.n_experts = n_experts
        self.n_experts, self.L, self.I = n_experts, L, I_
        self.safe = None

    def scan(self, stream=None):
        """Certify the experts for the tcgen05 kernels (one-time, synchronous)."""
        self.safe = torch.empty(self.n_experts, dtype=torch.uint8, device=self.bytes.device)
        check(lib.k3gpu_bank_scan(C.byref(self.desc), ptr(self.safe), stream_ptr(stream)),
              "k3gpu_bank_scan")
        return self.desc.n_f16_unsafe

    @staticmethod
    def layout(L, I_):
        d = K3GpuExpertBank()
        lib.k3gpu_bank_layout(C.byref(d), L, I_)
        return d


def moe_experts(z, idx, wt, bank: ExpertBank, topk, n_routed, n_shared, act, b1=4.0, b2=25.0,
                latent_norm=None, eps=1e-5, ws=None, stream=None):
    T, L = z.shape
    out = torch.empty((T, L), dtype=torch.float32, device=z.device)
    need = lib.k3gpu_moe_workspace(T, topk, n_shared, L, bank.I, n_routed)
    ws = ws if ws is not None else workspace(need, z.device)
    check(lib.k3gpu_moe_experts(ptr(out), ptr(z), ptr(idx), ptr(wt), C.byref(bank.desc), T, topk,
                                n_routed, n_shared, act, float(b1), float(b2), ptr(latent_norm),
                                float(eps), ptr(ws), ws.numel(), stream_ptr(stream)),
          "k3gpu_moe_experts")
    return out


def moe_experts_ptrs(out, z_ptr, idx_ptr, wt_ptr, T, bank: ExpertBank, topk, n_routed, n_shared, act, b1=4.0,
                     b2=25.0, ws=None, stream=None):
    """k3gpu_moe_experts on raw device pointers for the inputs (e.g. a peer-exchange
    arena's receive region); out is a [T][L] tensor."""
    need = lib.k3gpu_moe_workspace(T, topk, n_shared, bank.L, bank.I, n_routed)
    ws = ws if ws is not None else workspace(need, out.device)
    check(lib.k3gpu_moe_experts(ptr(out), z_ptr, idx_ptr, wt_ptr, C.byref(bank.desc), T, topk, n_routed,
                                n_shared, act, float(b1), float(b2), None, 1e-5, ptr(ws), ws.numel(),
                                stream_ptr(stream)), "k3gpu_moe_experts")
    return out


def moe_layer(x, gate_W, bias, bank: ExpertBank, topk, n_routed, n_shared, act, b1=4.0, b2=25.0,
              renorm=1, routed_scale=1.0, ws=None, out=None, idx=None, wt=None, stream=None):
    T, L = x.shape
    out = out if out is not None else torch.empty((T, L), dtype=torch.float32, device=x.device)
    idx = idx if idx is not None else torch.empty((T, topk), dtype=torch.int32, device=x.device)
    wt = wt if wt is not None else torch.empty((T, topk), dtype=torch.float32, device=x.device)
    need = lib.k3gpu_moe_workspace(T, topk, n_shared, L, bank.I, n_routed)
    ws = ws if ws is not None else workspace(need, x.device)
    check(lib.k3gpu_moe_layer(ptr(out), ptr(idx), ptr(wt), ptr(x), ptr(gate_W), ptr(bias),
                              C.byref(bank.desc), T, topk, n_routed, n_shared, act, float(b1),
                              float(b2), renorm, float(routed_scale), ptr(ws), ws.numel(),
                              stream_ptr(stream)), "k3gpu_moe_layer")
    return out, idx, wt


def moe_phase_timing(enable: bool) -> None:
    check(lib.k3gpu_moe_phase_timing(1 if enable else 0), "k3gpu_moe_phase_timing")


def moe_phase_ms():
    """[router, plan, gate/up, down, combine] device ms of the last MoE call."""
    buf = (F * 5)()
    n = lib.k3gpu_moe_phase_ms(buf, 5)
    if n < 0:
        check(n, "k3gpu_moe_phase_ms")
    return list(buf[:n])


# --------------------------------------------------------------------------- KDA ---
def kda_verify(state, q, k, v, alpha, beta, qscale, stream=None):
    B, T, H, D = q.shape
    o = torch.empty_like(q)
    check(lib.k3gpu_kda_verify(ptr(o), ptr(state), ptr(q), ptr(k), ptr(v), ptr(alpha), ptr(beta),
                               B, T, H, D, float(qscale), stream_ptr(stream)), "k3gpu_kda_verify")
    return o


def kda_verify_tree(state, q, k, v, alpha, beta, parent, qscale, stream=None):
    """k3gpu_kda_verify over a draft tree; parent int32 [T] (device)."""
    B, T, H, D = q.shape
    o = torch.empty_like(q)
    check(lib.k3gpu_kda_verify_tree(ptr(o), ptr(state), ptr(q), ptr(k), ptr(v), ptr(alpha), ptr(beta),
                                    ptr(parent), B, T, H, D, float(qscale), stream_ptr(stream)),
          "k3gpu_kda_verify_tree")
    return o


def kda_commit(state, k, v, alpha, beta, n, stream=None):
    B, T, H, D = k.shape
    check(lib.k3gpu_kda_commit(ptr(state), ptr(k), ptr(v), ptr(alpha), ptr(beta), ptr(n), B, T,
                               H, D, stream_ptr(stream)), "k3gpu_kda_commit")


def kda_prefill(state, q, k, v, alpha, beta, qscale, outputs=True, stream=None):
    """Read T positions into the carried state in place (chunked form); returns the
    outputs [B][T][H][D], or None with outputs=False."""
    B, T, H, D = q.shape
    o = torch.empty_like(q) if outputs else None
    check(lib.k3gpu_kda_prefill(ptr(state), ptr(o) if o is not None else None, ptr(q), ptr(k), ptr(v), ptr(alpha),
                                ptr(beta), B, T, H, D, float(qscale), stream_ptr(stream)), "k3gpu_kda_prefill")
    return o


def kda_prologue(q, k, v, z, b, q_conv, k_conv, v_conv, hist, A_log, dt_bias, H, D, K, lb,
                 stream=None):
    B, T, P = q.shape
    alpha = torch.empty_like(q)
    beta = torch.empty((B, T, H), dtype=torch.float32, device=q.device)
    pre = torch.empty((B, T, 3, P), dtype=torch.float32, device=q.device)
    check(lib.k3gpu_kda_prologue(ptr(q), ptr(k), ptr(v), ptr(alpha), ptr(beta), ptr(pre), ptr(z),
                                 ptr(b), ptr(q_conv), ptr(k_conv), ptr(v_conv), ptr(hist),
                                 ptr(A_log), ptr(dt_bias), B, T, H, D, K, float(lb),
                                 stream_ptr(stream)), "k3gpu_kda_prologue")
    return alpha, beta, pre


def kda_prologue_tree(q, k, v, z, b, q_conv, k_conv, v_conv, hist, A_log, dt_bias, parent, H, D, K, lb,
                      stream=None):
    """k3gpu_kda_prologue with each node's ShortConv window along its ancestors (parent
    int32 [T] device, or None: the chain)."""
    B, T, P = q.shape
    alpha = torch.empty_like(q)
    beta = torch.empty((B, T, H), dtype=torch.float32, device=q.device)
    pre = torch.empty((B, T, 3, P), dtype=torch.float32, device=q.device)
    check(lib.k3gpu_kda_prologue_tree(ptr(q), ptr(k), ptr(v), ptr(alpha), ptr(beta), ptr(pre), ptr(z),
                                      ptr(b), ptr(q_conv), ptr(k_conv), ptr(v_conv), ptr(hist),
                                      ptr(A_log), ptr(dt_bias), ptr(parent), B, T, H, D, K, float(lb),
                                      stream_ptr(stream)), "k3gpu_kda_prologue_tree")
    return alpha, beta, pre


def kda_commit_conv(hist, pre, n, H, D, K, stream=None):
    B, T = pre.shape[0], pre.shape[1]
    check(lib.k3gpu_kda_commit_conv(ptr(hist), ptr(pre), ptr(n), B, T, H, D, K,
                                    stream_ptr(stream)), "k3gpu_kda_commit_conv")


def kda_norm_gate(o, gate, o_norm, H, D, eps, stream=None):
    R = o.numel() // (H * D)
    check(lib.k3gpu_kda_norm_gate(ptr(o), ptr(gate), ptr(o_norm), R, H, D, float(eps),
                                  stream_ptr(stream)), "k3gpu_kda_norm_gate")


# --------------------------------------------------------------------------- MLA ---
def mla_absorbed(q_nope, q_rope, kv_b, lat, rope, cached, mask, v_head, max_ctx, scale,
                 ws=None, stream=None):
    B, T, H, qn = q_nope.shape
    qr = q_rope.shape[3]
    cap, kvl = lat.shape[1], lat.shape[2]
    out = torch.empty((B, T, H, v_head), dtype=torch.float32, device=q_nope.device)
    need = lib.k3gpu_mla_workspace(B, T, H, kvl, max_ctx)
    ws = ws if ws is not None else workspace(need, q_nope.device)
    check(lib.k3gpu_mla_absorbed(ptr(out), ptr(q_nope), ptr(q_rope), ptr(kv_b), ptr(lat),
                                 ptr(rope), ptr(cached), ptr(mask), B, T, H, qn, qr, v_head, kvl,
                                 cap, max_ctx, float(scale), ptr(ws), ws.numel(),
                                 stream_ptr(stream)), "k3gpu_mla_absorbed")
    return out


# ------------------------------------------------------------------------ accept ---
def accept_greedy(logits, drafts, nd_b=None, stream=None, arg=None):
    """Greedy chain acceptance from logits [B][nd+1][vocab], or, with logits None, from arg
    [B][nd+1] already holding every position's argmax (Model.verify(..., logits=False))."""
    if logits is None:
        B, T = arg.shape
        V, dev = 0, arg.device
    else:
        B, T, V = logits.shape
        dev = logits.device
        arg = torch.empty((B, T), dtype=torch.int32, device=dev)
    nd = T - 1
    emit = torch.empty((B, T), dtype=torch.int32, device=dev)
    n_emit = torch.empty((B,), dtype=torch.int32, device=dev)
    check(lib.k3gpu_accept_greedy(ptr(emit), ptr(n_emit), ptr(arg), ptr(logits), ptr(drafts),
                                  ptr(nd_b), B, nd, V, stream_ptr(stream)), "k3gpu_accept_greedy")
    return emit, n_emit, arg


def accept_tree_greedy(logits, tok, parent, stream=None, arg=None):
    """Greedy acceptance over a draft tree from logits [B][T][vocab], or, with logits None,
    from arg [B][T] already holding every node's argmax (Model.verify(..., logits=False))."""
    if logits is None:
        B, T = arg.shape
        V, dev = 0, arg.device
    else:
        B, T, V = logits.shape
        dev = logits.device
        arg = torch.empty((B, T), dtype=torch.int32, device=dev)
    emit = torch.empty((B, T), dtype=torch.int32, device=dev)
    path = torch.empty((B, T), dtype=torch.int32, device=dev)
    n_emit = torch.empty((B,), dtype=torch.int32, device=dev)
    check(lib.k3gpu_accept_tree_greedy(ptr(emit), ptr(n_emit), ptr(path), ptr(arg), ptr(logits),
                                       ptr(tok), ptr(parent), B, T, V, stream_ptr(stream)),
          "k3gpu_accept_tree_greedy")
    return emit, n_emit, path, arg


# ------------------------------------------------------------ trunk matmul ---------
def matmul_bf16(X, W, out=None, ws=None, stream=None):
    """k3_matmul_bf16_batch: Y [T][out] = X [T][in] . W^T with W bf16 [out][in]
    (torch.bfloat16 or int16/uint16 bit patterns). X and Y may be row slices of wider
    tensors (their row strides are passed as ldx / ldy)."""
    T, n_in = X.shape
    n_out = W.shape[0]
    Y = out if out is not None else torch.empty((T, n_out), dtype=torch.float32, device=X.device)
    need = lib.k3gpu_matmul_bf16_workspace(T, n_in, n_out)
    ws = ws if ws is not None else workspace(need, X.device)
    check(lib.k3gpu_matmul_bf16_batch(Y.data_ptr(), Y.stride(0), X.data_ptr(), X.stride(0), ptr(W), n_in,
                                      n_out, T, ptr(ws), ws.numel(), stream_ptr(stream)),
          "k3gpu_matmul_bf16_batch")
    return Y


def lm_head_argmax(X, W, ws=None, stream=None):
    """The lm_head fused with the greedy argmax: arg int32 [T] = first index of the maximum
    of X [T][in] . W^T (W bf16 [vocab][in]) over non-NaN values, 0 when the value at index
    0 is NaN; the logits are never written."""
    T, n_in = X.shape
    vocab = W.shape[0]
    arg = torch.empty(T, dtype=torch.int32, device=X.device)
    need = lib.k3gpu_lm_head_argmax_workspace(T, n_in, vocab)
    ws = ws if ws is not None else workspace(need, X.device)
    check(lib.k3gpu_lm_head_argmax(arg.data_ptr(), X.data_ptr(), X.stride(0), ptr(W), n_in, vocab, T, ptr(ws),
                                   ws.numel(), stream_ptr(stream)), "k3gpu_lm_head_argmax")
    return arg


# ------------------------------------------------------------- decoder layer -------
def layer_cfg(**kw) -> K3GpuLayerCfg:
    c = K3GpuLayerCfg()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def kda_weights(w: dict) -> K3GpuKdaW:
    """w: q, k, v, b, f_a, f_b, g, o (bf16 bit tensors [out][in]), q_conv, k_conv, v_conv,
    A_log, dt_bias, o_norm (fp32) -- CUDA tensors, kept alive by the caller."""
    kw = K3GpuKdaW()
    for n, _ in K3GpuKdaW._fields_:
        setattr(kw, n, ptr(w[n]))
    return kw


def kda_log(B, T, H, D, device="cuda"):
    P = H * D
    z = lambda *s: torch.empty(s, dtype=torch.float32, device=device)
    t = {"k": z(B, T, P), "v": z(B, T, P), "alpha": z(B, T, P), "beta": z(B, T, H), "pre": z(B, T, 3, P)}
    lg = K3GpuKdaLog(*(ptr(t[n]) for n, _ in K3GpuKdaLog._fields_))
    return lg, t


def kda_layer_verify(x, w: dict, cfg: K3GpuLayerCfg, state, conv_hist, B, T, stream=None):
    """k3_kda_layer_log for B sequences: x [B*T][E] -> (out [B*T][E], log tensors)."""
    out = torch.empty_like(x)
    kw = kda_weights(w)
    lg, lt = kda_log(B, T, cfg.kda_heads, cfg.kda_head_dim, x.device)
    ws = workspace(lib.k3gpu_kda_layer_workspace(C.byref(cfg), B, T), x.device)
    check(lib.k3gpu_kda_layer_verify(ptr(out), ptr(x), C.byref(kw), C.byref(cfg), ptr(state), ptr(conv_hist),
                                     C.byref(lg), B, T, ptr(ws), ws.numel(), stream_ptr(stream)),
          "k3gpu_kda_layer_verify")
    return out, lt


def moe_weights(w: dict, bank: "ExpertBank") -> K3GpuMoeW:
    """w: down, up, sh1, sh3, sh2 (bf16 bit tensors; the sh* may be absent), gate_W,
    gate_bias, latent_norm (may be absent) -- CUDA tensors kept alive by the caller."""
    mw = K3GpuMoeW()
    for n in ("down", "up", "sh1", "sh3", "sh2", "gate_W", "gate_bias", "latent_norm"):
        setattr(mw, n, ptr(w.get(n)))
    mw.bank = C.pointer(bank.desc)
    return mw


def moe_prefill(x, w: dict, bank: "ExpertBank", cfg: K3GpuMoeCfg, stream=None):
    """The K3 MoE block (k3_moe_prefill): x [T][E] -> (out [T][E], idx, wt)."""
    T = x.shape[0]
    out = torch.empty_like(x)
    idx = torch.empty((T, cfg.topk), dtype=torch.int32, device=x.device)
    wt = torch.empty((T, cfg.topk), dtype=torch.float32, device=x.device)
    mw = moe_weights(w, bank)
    ws = workspace(lib.k3gpu_moe_prefill_workspace(C.byref(cfg), T), x.device)
    check(lib.k3gpu_moe_prefill(ptr(out), ptr(idx), ptr(wt), ptr(x), C.byref(mw), C.byref(cfg), T, ptr(ws),
                                ws.numel(), stream_ptr(stream)), "k3gpu_moe_prefill")
    return out, idx, wt


def decoder_layer_kda_verify(h, block_residual, n_blocks, w: dict, bank: "ExpertBank", cfg: K3GpuLayerCfg,
                             layer_idx, state, conv_hist, B, T, moe: dict = None, stream=None):
    """k3_decoder_layer_inc_log for a KDA + MoE layer, in place on h [B*T][E];
    block_residual [B*T][maxb][E] and n_blocks int32 [B*T] are updated on a boundary layer.
    Returns (moe idx, moe wt, log tensors)."""
    lw = K3GpuKdaLayerW()
    for n in ("attn_res_fold", "mlp_res_fold", "in_norm", "post_norm", "gate_W", "gate_bias"):
        setattr(lw, n, ptr(w[n]))
    lw.kda = kda_weights(w)
    lw.bank = C.pointer(bank.desc)
    if moe is not None:                      # the K3 MoE form; `bank` then holds the latent experts
        mw = moe_weights(moe, bank)
        lw.moe = C.pointer(mw)
    R = B * T
    idx = torch.empty((R, cfg.topk), dtype=torch.int32, device=h.device)
    wt = torch.empty((R, cfg.topk), dtype=torch.float32, device=h.device)
    lg, lt = kda_log(B, T, cfg.kda_heads, cfg.kda_head_dim, h.device)
    ws = workspace(lib.k3gpu_decoder_layer_workspace(C.byref(cfg), B, T), h.device)
    check(lib.k3gpu_decoder_layer_kda_verify(ptr(h), ptr(block_residual), ptr(n_blocks), ptr(idx), ptr(wt),
                                             C.byref(lw), C.byref(cfg), layer_idx, ptr(state), ptr(conv_hist),
                                             C.byref(lg), B, T, ptr(ws), ws.numel(), stream_ptr(stream)),
          "k3gpu_decoder_layer_kda_verify")
    return idx, wt, lt


def mla_weights(w: dict) -> K3GpuMlaW:
    """w: q_a, q_b, kv_a, g (or absent / None: no gate), o (bf16 bit tensors [out][in]),
    q_a_norm, kv_a_norm, kv_b (fp32) -- CUDA tensors, kept alive by the caller."""
    mw = K3GpuMlaW()
    for n, _ in K3GpuMlaW._fields_:
        setattr(mw, n, ptr(w.get(n)))
    return mw


def mla_layer_verify(x, w: dict, cfg: K3GpuLayerCfg, lat, rope, cached, mask, max_ctx, B, T, stream=None):
    """k3_mla_cached (absorbed latent layout) for B sequences of T query nodes: x [B*T][E] ->
    out [B*T][E]; the new rows are appended to lat [B][cap][kv_lora] / rope [B][cap][qk_rope]
    (bf16 bits) at cached[b] + t. cached int32 [B], mask int64 [T] (device)."""
    mw = mla_weights(w)
    out = torch.empty_like(x)
    cap = lat.shape[1]
    ws = workspace(lib.k3gpu_mla_layer_workspace(C.byref(cfg), B, T, max_ctx), x.device)
    check(lib.k3gpu_mla_layer_verify(ptr(out), ptr(x), C.byref(mw), C.byref(cfg), ptr(lat), ptr(rope), cap,
                                     ptr(cached), ptr(mask), max_ctx, B, T, ptr(ws), ws.numel(), stream_ptr(stream)),
          "k3gpu_mla_layer_verify")
    return out


def decoder_layer_mla_verify(h, block_residual, n_blocks, w: dict, bank: "ExpertBank", cfg: K3GpuLayerCfg,
                             layer_idx, lat, rope, cached, mask, max_ctx, B, T, moe: dict = None, stream=None):
    """k3_decoder_layer_inc_log for an MLA + MoE layer, in place on h [B*T][E] (cache
    arguments as mla_layer_verify). Returns (moe idx, moe wt)."""
    lw = K3GpuMlaLayerW()
    for n in ("attn_res_fold", "mlp_res_fold", "in_norm", "post_norm", "gate_W", "gate_bias"):
        setattr(lw, n, ptr(w[n]))
    lw.mla = mla_weights(w)
    lw.bank = C.pointer(bank.desc)
    if moe is not None:
        mw = moe_weights(moe, bank)
        lw.moe = C.pointer(mw)
    R = B * T
    idx = torch.empty((R, cfg.topk), dtype=torch.int32, device=h.device)
    wt = torch.empty((R, cfg.topk), dtype=torch.float32, device=h.device)
    cap = lat.shape[1]
    ws = workspace(lib.k3gpu_decoder_layer_mla_workspace(C.byref(cfg), B, T, max_ctx), h.device)
    check(lib.k3gpu_decoder_layer_mla_verify(ptr(h), ptr(block_residual), ptr(n_blocks), ptr(idx), ptr(wt),
                                             C.byref(lw), C.byref(cfg), layer_idx, ptr(lat), ptr(rope), cap,
                                             ptr(cached), ptr(mask), max_ctx, B, T, ptr(ws), ws.numel(),
                                             stream_ptr(stream)),
          "k3gpu_decoder_layer_mla_verify")
    return idx, wt


# ----------------------------------------------------------------- norms ---------
def rmsnorm(x, w, eps, out=None, stream=None):
    """k3_rmsnorm over the rows of x [T][n]."""
    T, n = x.shape
    y = out if out is not None else torch.empty_like(x)
    check(lib.k3gpu_rmsnorm(ptr(y), ptr(x), ptr(w), T, n, float(eps), stream_ptr(stream)), "k3gpu_rmsnorm")
    return y


def attn_res(block_residual, cur, fold, n_blocks, eps, stream=None):
    """k3_attn_res per position: sources block_residual[t][:n_blocks[t]] then cur[t].
    block_residual [T][maxb][n] (maxb may be 0: pass None), cur [T][n], n_blocks int32 [T]."""
    T, n = cur.shape
    maxb = 0 if block_residual is None else block_residual.shape[1]
    out = torch.empty_like(cur)
    check(lib.k3gpu_attn_res(ptr(out), ptr(block_residual), ptr(cur), ptr(fold), ptr(n_blocks), T,
                             maxb, n, float(eps), stream_ptr(stream)), "k3gpu_attn_res")
    return out


def accept_sample(logits, drafts, temp, seed, offset=0, nd_b=None, stream=None):
    B, T, V = logits.shape
    nd = T - 1
    emit = torch.full((B, T), -1, dtype=torch.int32, device=logits.device)
    n_emit = torch.empty((B,), dtype=torch.int32, device=logits.device)
    check(lib.k3gpu_accept_sample(ptr(emit), ptr(n_emit), ptr(logits), ptr(drafts), ptr(nd_b), B,
                                  nd, V, float(temp), int(seed), int(offset), stream_ptr(stream)),
          "k3gpu_accept_sample")
    return emit, n_emit


# ----------------------------------------------------------------------- drafter ---
def spec_draft(seq, cap=8, nmax=4, nmin=3):
    arr = (C.c_int * max(len(seq), 1))(*seq)
    out = (C.c_int * max(cap, 1))()
    nd = lib.k3_spec_draft_ngram(arr, len(seq), cap, nmax, nmin, out)
    return list(out[:nd])


def bank_read_safetensors(files, layer, e0, n, L, I_):
    """Routed experts [e0, e0 + n) of a MoE layer from safetensors shards into a host
    uint8 array in the device bank layout (k3_bank_read_safetensors); upload it with one
    copy (e.g. torch.from_numpy(...).cuda()) and wrap it in an ExpertBank."""
    import numpy as np
    lay = ExpertBank.layout(L, I_)
    buf = np.zeros(n * lay.stride, np.uint8)
    arr = (C.c_char_p * len(files))(*[os.fsencode(f) for f in files])
    check(lib.k3_bank_read_safetensors(arr, len(files), layer, e0, n, L, I_, buf.ctypes.data, buf.nbytes),
          "k3_bank_read_safetensors")
    return buf


def spec_draft_eager(seq, cap=8):
    """The drafting study's P1 (k3_spec_draft_eager): host C, no GPU."""
    arr = (C.c_int * max(len(seq), 1))(*seq)
    out = (C.c_int * max(cap, 1))()
    nd = lib.k3_spec_draft_eager(arr, len(seq), cap, out)
    return list(out[:nd])


def _p3_table(q):
    q = [float(v) for v in q]
    if len(q) != SPEC_P3_CODES:
        raise ValueError(f"a P3 acceptance table has {SPEC_P3_CODES} entries, got {len(q)}")
    return (C.c_double * SPEC_P3_CODES)(*q)


def spec_p3_length(codes, q, delta, cumulative=True) -> int:
    """The study's adaptive_lengths for one draft point (k3_spec_p3_length)."""
    codes = list(codes)
    arr = (C.c_ubyte * max(len(codes), 1))(*codes)
    return lib.k3_spec_p3_length(arr, len(codes), _p3_table(q), float(delta), int(bool(cumulative)))


def spec_p3_cost_length(codes, q, cost, replay=False) -> int:
    """The study's cost_aware_lengths for one draft point (k3_spec_p3_cost_length)."""
    codes = list(codes)
    arr = (C.c_ubyte * max(len(codes), 1))(*codes)
    return lib.k3_spec_p3_cost_length(arr, len(codes), _p3_table(q), C.byref(cost), int(bool(replay)))


class SuffixDrafter:
    """The drafting study's P2 as an incremental host drafter (k3_suffix_drafter_*): push
    ids as they are accepted, draft() after each step. No GPU."""

    def __init__(self, capacity: int):
        self._d = lib.k3_suffix_drafter_create(capacity)
        if not self._d:
            raise K3Error(f"k3_suffix_drafter_create({capacity}) failed")

    def push(self, ids) -> None:
        ids = list(ids)
        arr = (C.c_int * max(len(ids), 1))(*ids)
        check(lib.k3_suffix_drafter_push(self._d, arr, len(ids)), "k3_suffix_drafter_push")

    def __len__(self) -> int:
        return lib.k3_suffix_drafter_length(self._d)

    def draft(self, cap=8, min_len=1):
        """(draft ids, match length, period); the draft is empty when the longest earlier
        match is shorter than min_len."""
        out = (C.c_int * max(cap, 1))()
        L, g = C.c_int(0), C.c_int(0)
        nd = lib.k3_suffix_drafter_draft(self._d, cap, min_len, out, C.byref(L), C.byref(g))
        return list(out[:nd]), L.value, g.value

    def tree(self, max_nodes=64, branch=4, max_depth=8, min_len=1):
        """(tok, parent) of a draft tree rooted at the pending id (k3_suffix_drafter_tree)."""
        tok = (C.c_int * max_nodes)()
        par = (C.c_int * max_nodes)()
        n = lib.k3_suffix_drafter_tree(self._d, max_nodes, branch, max_depth, min_len, tok, par)
        return list(tok[:n]), list(par[:n])

    def features(self, draft):
        """P3 feature codes of `draft` continuing the history (k3_suffix_drafter_features);
        255 at every position when the history has no earlier match."""
        draft = list(draft)
        arr = (C.c_int * max(len(draft), 1))(*draft)
        codes = (C.c_ubyte * max(len(draft), 1))()
        check(lib.k3_suffix_drafter_features(self._d, arr, len(draft), codes), "k3_suffix_drafter_features")
        return list(codes[:len(draft)])

    def draft_p3(self, q, delta=0.22, cost=None, replay=False, cap=8):
        """The P3 draft: P2's draft cut by the acceptance table q (delta rule, or the cost
        rule when `cost` is a K3SpecCost)."""
        qa = _p3_table(q)
        out = (C.c_int * max(cap, 1))()
        nd = lib.k3_suffix_drafter_draft_p3(self._d, qa, float(delta), C.byref(cost) if cost is not None else None,
                                            int(bool(replay)), cap, out)
        return list(out[:nd])

    def close(self) -> None:
        if self._d:
            lib.k3_suffix_drafter_free(self._d)
            self._d = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown may have unloaded the library
            pass


def layer_loop_plan(n_layers, attn_res_block, loop_count, span=None, preset=False):
    """(vmap, (A, B), attn_res_extra) of the layer loop (k3_layer_loop_plan): the physical
    layer executed at each position, each position owning its own state slot."""
    a, b = span if span is not None else (0, 0)
    cap = n_layers * max(loop_count, 1)
    vmap = (C.c_int * cap)()
    sp = (C.c_int * 2)()
    extra = C.c_int(0)
    nv = lib.k3_layer_loop_plan(n_layers, attn_res_block, int(bool(preset)), a, b, loop_count, vmap, cap, sp,
                                C.byref(extra))
    check(nv if nv < 0 else 0, "k3_layer_loop_plan")
    return list(vmap[:nv]), (sp[0], sp[1]), extra.value


class SpecLoop:
    """The engine's speculative decode loop (k3_spec_loop_*): host bookkeeping over two
    callables, verify(ids, base, parent) -> the model's next id after each fed node
    (parent None for a chain), and commit(base, keep, path) (path None: the first keep
    positions; else the accepted tree nodes). With device ops behind them it drives the
    verify forward; on the host it drives any model."""

    def __init__(self, ids, verify, commit, *, cached=0, policy=DRAFT_NGRAM, spec_n=8, min_len=1, gen=64,
                 tmax=None, kv_cap=None, stop_ids=(), p3_q=None, p3_delta=0.22, p3_cost=None, p3_replay=False,
                 tree_nodes=64, tree_branch=4, draft_verify=None, draft_commit=None, prefill_chunk=0,
                 pause_after=0, checkpoint=None, native=None):
        ids = [int(v) for v in ids]
        tmax = tmax if tmax is not None else len(ids) + gen + 1
        self._errors = []

        def _verify(_ctx, p, par, n, base, arg):
            try:
                out = verify([p[i] for i in range(n)], base, [par[i] for i in range(n)] if par else None)
                if len(out) != n:
                    raise ValueError(f"verify returned {len(out)} ids for {n} positions")
                for i, v in enumerate(out):
                    arg[i] = int(v)
                return 0
            except Exception as e:  # noqa: BLE001 -- reported by step()
                self._errors.append(e)
                return 1

        def _commit(_ctx, base, path, keep):
            try:
                commit(base, keep, [path[i] for i in range(keep)] if path else None)
                return 0
            except Exception as e:  # noqa: BLE001
                self._errors.append(e)
                return 1

        def wrap_verify(fn):
            def _cb(_ctx, p, par, n, base, arg):
                try:
                    out = fn([p[i] for i in range(n)], base, [par[i] for i in range(n)] if par else None)
                    if len(out) != n:
                        raise ValueError(f"verify returned {len(out)} ids for {n} positions")
                    for i, v in enumerate(out):
                        arg[i] = int(v)
                    return 0
                except Exception as e:  # noqa: BLE001 -- reported by step()
                    self._errors.append(e)
                    return 1
            return _cb

        def wrap_commit(fn):
            def _cb(_ctx, base, path, keep):
                try:
                    fn(base, keep, [path[i] for i in range(keep)] if path else None)
                    return 0
                except Exception as e:  # noqa: BLE001
                    self._errors.append(e)
                    return 1
            return _cb

        self._L = None
        self._fns = (SpecVerifyFn(_verify), SpecCommitFn(_commit))
        if draft_verify is not None:
            self._fns += (SpecVerifyFn(wrap_verify(draft_verify)), SpecCommitFn(wrap_commit(draft_commit)))
        self._stop = (C.c_int * max(len(stop_ids), 1))(*stop_ids)
        self._q = _p3_table(p3_q) if p3_q is not None else None
        self._cost = p3_cost
        cfg = K3SpecLoopCfg(policy, spec_n, min_len, gen, tmax, kv_cap if kv_cap is not None else tmax,
                            C.cast(self._stop, VP), len(stop_ids), C.cast(self._q, VP) if self._q else None,
                            float(p3_delta), C.cast(C.pointer(p3_cost), VP) if p3_cost is not None else None,
                            int(bool(p3_replay)), tree_nodes, tree_branch, prefill_chunk, pause_after)
        arr = (C.c_int * max(len(ids), 1))(*ids)
        if native is not None:     # C callbacks (e.g. k3gpu_model_loop_verify / _commit) and their ctx
            vfn, cfn, ctx = native
            self._native = native
            self._L = lib.k3_spec_loop_create(C.byref(cfg), arr, len(ids), cached, C.cast(vfn, VP),
                                              C.cast(cfn, VP), ctx)
        else:
            self._L = lib.k3_spec_loop_create(C.byref(cfg), arr, len(ids), cached,
                                              C.cast(self._fns[0], VP), C.cast(self._fns[1], VP), None)
        if not self._L:
            raise K3Error("k3_spec_loop_create: bad configuration")
        if draft_verify is not None:
            check(lib.k3_spec_loop_set_draft_model(self._L, C.cast(self._fns[2], VP), C.cast(self._fns[3], VP), None),
                  "k3_spec_loop_set_draft_model")
        if checkpoint is not None:
            def _ck(_ctx, cached):
                try:
                    checkpoint(cached)
                    return 0
                except Exception as e:  # noqa: BLE001
                    self._errors.append(e)
                    return 1
            self._ckfn = SpecCheckpointFn(_ck)
            check(lib.k3_spec_loop_set_checkpoint(self._L, C.cast(self._ckfn, VP), None), "k3_spec_loop_set_checkpoint")
        self.tmax = tmax

    def step(self):
        """(ids kept this step, trace dict); ([], None) once finished."""
        out = (C.c_int * 9)()
        n = C.c_int(0)
        tr = K3SpecStepTrace()
        st = lib.k3_spec_loop_step(self._L, out, C.byref(n), C.byref(tr))
        if st < 0:
            err = self._errors.pop() if self._errors else None
            raise K3Error(f"k3_spec_loop_step: {lib.k3gpu_strerror(st).decode()}") from err
        if st > 0:
            return [], None
        return list(out[:n.value]), {"nd": tr.nd, "m": tr.m, "keep": tr.keep, "fed": tr.fed}

    def request_pause(self):
        """Pause the prompt read-in at its next checkpoint (the engine's SIGINT)."""
        lib.k3_spec_loop_request_pause(self._L)

    def run(self):
        """Step until finished; returns (generated ids, per-step traces)."""
        gen, traces = [], []
        while True:
            ids, tr = self.step()
            if tr is None:
                return gen, traces
            gen += ids
            traces.append(tr)

    def state(self):
        T, cached, nout = C.c_int(0), C.c_int(0), C.c_int(0)
        s = K3SpecLoopStats()
        done = lib.k3_spec_loop_state(self._L, C.byref(T), C.byref(cached), C.byref(nout), C.byref(s))
        stats = {f: getattr(s, f) for f, _ in K3SpecLoopStats._fields_ if f != "hist"}
        stats["hist"] = list(s.hist)
        return {"T": T.value, "cached": cached.value, "nout": nout.value, "done": done, "stats": stats}

    def ids(self):
        buf = (C.c_int * self.tmax)()
        T = lib.k3_spec_loop_ids(self._L, buf, self.tmax)
        return list(buf[:T])

    def close(self) -> None:
        if self._L:
            lib.k3_spec_loop_free(self._L)
            self._L = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown may have unloaded the library
            pass


class SafetensorsIndex:
    """A checkpoint's shards indexed by tensor name (k3_st_open / find / read): host C, no
    GPU. Open a directory (every *.safetensors in it) or a list of shard paths."""

    _NP = {ST_U8: "uint8", ST_BF16: "uint16", ST_F16: "float16", ST_F32: "float32"}

    def __init__(self, where):
        if isinstance(where, (str, bytes, os.PathLike)):
            self._s = lib.k3_st_open(os.fsencode(where))
        else:
            paths = [os.fsencode(p) for p in where]
            arr = (C.c_char_p * max(len(paths), 1))(*paths)
            self._s = lib.k3_st_open_files(arr, len(paths))
        if not self._s:
            raise K3Error(f"k3_st_open: cannot index {where!r}")

    def names(self):
        return [lib.k3_st_name(self._s, i).decode() for i in range(lib.k3_st_count(self._s))]

    def info(self, name):
        t = K3StTensorInfo()
        check(lib.k3_st_find(self._s, name.encode(), C.byref(t)), f"k3_st_find({name!r})")
        return {"dtype": t.dtype, "dtype_name": t.dtype_name.decode(), "shape": list(t.shape[:t.ndim]),
                "shard": t.shard, "nbytes": t.nbytes}

    def read(self, name):
        """The stored bytes as a numpy array of the tensor's shape (bf16 as uint16 bit
        patterns; other dtypes as raw uint8)."""
        import numpy as np
        t = self.info(name)
        buf = np.empty(t["nbytes"], np.uint8)
        got = lib.k3_st_read(self._s, name.encode(), buf.ctypes.data, buf.nbytes)
        check(int(got) if got < 0 else 0, f"k3_st_read({name!r})")
        dt = self._NP.get(t["dtype"])
        return buf.view(dt).reshape(t["shape"]) if dt else buf

    def close(self) -> None:
        if self._s:
            lib.k3_st_close(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown may have unloaded the library
            pass


# ------------------------------------------------------------ model verify forward --
def _sibling(name):
    """A module of this package by file (the directory name is not an identifier)."""
    import importlib.util
    import sys
    key = f"{__name__}_{name}"
    if key not in sys.modules:
        spec = importlib.util.spec_from_file_location(key, os.path.join(PKG, name + ".py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[key] = mod
        spec.loader.exec_module(mod)
    return sys.modules[key]


def launch_count() -> int:
    """The library's kernel launches so far in this process (k3gpu_launch_count)."""
    return int(lib.k3gpu_launch_count())


def argmax(logits, stream=None):
    """argmax_ per row of logits [rows][vocab] on the device (int32 [rows])."""
    rows, V = logits.reshape(-1, logits.shape[-1]).shape
    arg = torch.empty(rows, dtype=torch.int32, device=logits.device)
    check(lib.k3gpu_argmax(ptr(arg), ptr(logits), rows, V, stream_ptr(stream)), "k3gpu_argmax")
    return arg


class Model:
    """A whole K3-architecture model on the device: the verify forward of k3gpu_model_*
    (embed, every KDA/MLA + MoE decoder layer, the model-level AttnRes, the final norm, the
    lm_head and the per-position argmax over B sequences) and its commit.

    Built from a checkpoint directory (config.json + safetensors shards, the released
    layout) with the package's config reader, tensor index and binder; the routed experts
    of every MoE layer are read by k3_bank_read_safetensors into one device bank per layer.
    Or from already bound fields (`from_fields`), for synthetic weights made on the device.
    The model's state (KDA states and logs, MLA caches, activations) lives in one arena
    this object allocates with torch; every computation runs in the library's kernels."""

    def __init__(self, cfg: dict, layers: list, top: dict, banks: list, B=1, max_T=64, kv_cap=1024,
                 device="cuda", stream=None):
        n = cfg["num_hidden_layers"]
        if cfg.get("first_k_dense_replace", 0) > 0:
            raise K3Error("dense MLP layers (first_k_dense_replace > 0) are not on the verify path")
        self.cfg, self.B, self.max_T, self.kv_cap = cfg, B, max_T, kv_cap
        self.device = torch.device(device)
        self.stream = stream
        self.vocab = cfg["vocab_size"]
        self._alive = [layers, top, banks]
        cm = _sibling("config")
        self.lcfg = cm.layer_cfg(sys_module(), cfg)
        # "plain": the benchmark configurations' MoE (router and experts at the hidden width,
        # the shared experts in the same bank, SwiGLU); otherwise the K3 LatentMoE form
        plain = cfg.get("moe_form", "latent") == "plain"
        if plain:
            self.lcfg.latent, self.lcfg.shared_inter = 0, 0
            self.lcfg.act = ACT_SWIGLU if cfg.get("act", "swiglu") == "swiglu" else ACT_SITU
        self._kda = (K3GpuKdaLayerW * n)()
        self._mla = (K3GpuMlaLayerW * n)()
        self._moe = []
        self._is_mla = (C.c_int * n)()
        use_norm = cfg.get("latent_moe_use_norm", True)
        for L in range(n):
            d, bank = layers[L], banks[L]
            mw = None
            if not plain:
                mw = K3GpuMoeW()
                for f in ("down", "up", "sh1", "sh3", "sh2", "gate_W", "gate_bias"):
                    setattr(mw, f, ptr(d.get(f)))
                mw.latent_norm = ptr(d["latent_norm"]) if use_norm else None
                mw.bank = C.pointer(bank.desc)
                self._moe.append(mw)
            mla = d["kind"] == "mla"
            self._is_mla[L] = int(mla)
            lw = self._mla[L] if mla else self._kda[L]
            for f in ("attn_res_fold", "mlp_res_fold", "in_norm", "post_norm", "gate_W", "gate_bias"):
                setattr(lw, f, ptr(d[f]))
            if mla:
                lw.mla = mla_weights(d)
            else:
                lw.kda = kda_weights(d)
            lw.bank = C.pointer(bank.desc)
            lw.moe = C.pointer(mw) if mw is not None else None
        self._c = K3GpuModelCfg(self.lcfg, n, self.vocab, C.cast(self._is_mla, VP))
        self._w = K3GpuModelW(ptr(top["embed"]), ptr(top["lm_head"]), ptr(top["norm"]),
                              ptr(top.get("out_res_fold")), self._kda, self._mla)
        need = lib.k3gpu_model_arena_bytes(C.byref(self._c), B, max_T, kv_cap)
        if need == 0:
            raise K3Error("k3gpu_model_arena_bytes: configuration refused")
        self.arena = torch.empty(need + 256, dtype=torch.uint8, device=self.device)
        base = (self.arena.data_ptr() + 255) & ~255
        self._m = lib.k3gpu_model_create(C.byref(self._c), C.byref(self._w), B, max_T, kv_cap, VP(base), need,
                                         stream_ptr(stream))
        if not self._m:
            raise K3Error("k3gpu_model_create failed")
        self.arena_bytes = need

    @classmethod
    def from_checkpoint(cls, ckpt_dir, B=1, max_T=64, kv_cap=1024, device="cuda", stream=None, scan=True):
        import glob
        cm, bm = _sibling("config"), _sibling("bind")
        cfg = cm.read_config(os.path.join(ckpt_dir, "config.json"))
        index = SafetensorsIndex(ckpt_dir)
        binder = bm.Binder(index, cfg)
        files = sorted(glob.glob(os.path.join(ckpt_dir, "*.safetensors")))
        n_exp, Lt, I_ = cfg["num_experts"], cfg["routed_expert_hidden_size"], cfg["moe_intermediate_size"]
        layers, banks = [], []
        for L in range(cfg["num_hidden_layers"]):
            f = binder.layer(L)
            d = bm.to_device(f, device)
            d["kind"] = f["kind"]
            if f["kind"] == "mla" and f.get("g") is None:
                d["g"] = None
            layers.append(d)
            host = bank_read_safetensors(files, L, 0, n_exp, Lt, I_)
            bank = ExpertBank(torch.from_numpy(host).to(device), n_exp, Lt, I_)
            if scan:
                bank.scan(stream)
            banks.append(bank)
        top = bm.to_device(binder.model(), device)
        index.close()
        return cls(cfg, layers, top, banks, B=B, max_T=max_T, kv_cap=kv_cap, device=device, stream=stream)

    def close(self):
        if getattr(self, "_m", None):
            lib.k3gpu_model_free(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown may have unloaded the library
            pass

    def reset(self):
        check(lib.k3gpu_model_reset(self._m), "k3gpu_model_reset")

    def verify(self, ids, parent=None, logits=True):
        """ids int32 [B][T] (device) -> (arg int32 [B][T], logits view [B][T][vocab]);
        parent: host list [T] (a draft tree shared by the sequences) or None (a chain).
        The logits view is the model's own buffer, valid until the next sweep. logits=False:
        the lm_head fused with the argmax (greedy acceptance needs no logits) -> (arg, None)."""
        ids = ids.to(self.device, torch.int32).contiguous()
        B, T = ids.shape
        arg = torch.empty((B, T), dtype=torch.int32, device=self.device)
        par = (C.c_int * T)(*parent) if parent is not None else None
        if not logits:
            check(lib.k3gpu_model_verify_greedy(self._m, ptr(ids), T, par, ptr(arg)), "k3gpu_model_verify_greedy")
            return arg, None
        lp = VP()
        check(lib.k3gpu_model_verify(self._m, ptr(ids), T, par, ptr(arg), C.byref(lp)), "k3gpu_model_verify")
        return arg, self.logits_view(lp.value, B, T)

    def logits_view(self, addr, B, T):
        off = addr - self.arena.data_ptr()
        n = B * T * self.vocab
        return self.arena[off:off + 4 * n].view(torch.float32).view(B, T, self.vocab)

    def commit(self, keep, path=None):
        """keep: host ints [B]; path: host [B][T] accepted tree nodes (tree sweeps only)."""
        kk = (C.c_int * self.B)(*[int(v) for v in keep])
        pp = None
        if path is not None:
            flat = [int(v) for row in path for v in row]
            pp = (C.c_int * len(flat))(*flat)
        check(lib.k3gpu_model_commit(self._m, kk, pp), "k3gpu_model_commit")

    def prefill(self, ids):
        """ids int32 [B][n] (device): read in and committed; returns the next ids [B]."""
        ids = ids.to(self.device, torch.int32).contiguous()
        nxt = torch.empty(self.B, dtype=torch.int32, device=self.device)
        check(lib.k3gpu_model_prefill(self._m, ptr(ids), ids.shape[1], ptr(nxt)), "k3gpu_model_prefill")
        return nxt

    def set_cached(self, cached):
        """Positions consumed per sequence (host ints [B]), after writing states and cache
        rows through kda_state / mla_cache (a resumed session)."""
        c = (C.c_int * self.B)(*[int(v) for v in cached])
        check(lib.k3gpu_model_set_cached(self._m, c), "k3gpu_model_set_cached")

    def cached(self):
        c = (C.c_int * self.B)()
        check(lib.k3gpu_model_cached(self._m, c), "k3gpu_model_cached")
        return list(c)

    def last_routing(self, T):
        """The last layer's routing of the last sweep of T positions: int32 [B*T][topk] view."""
        p = VP()
        check(lib.k3gpu_model_last_routing(self._m, C.byref(p)), "k3gpu_model_last_routing")
        return self._view(p.value, (self.B * T, self.lcfg.topk), torch.int32)

    def kda_state(self, layer):
        """(state [B][H][D][D], conv history [B][3][P][K-1]) device views of a KDA layer."""
        st, hi = VP(), VP()
        check(lib.k3gpu_model_kda_state(self._m, layer, C.byref(st), C.byref(hi)), "k3gpu_model_kda_state")
        c = self.lcfg
        H, D, K = c.kda_heads, c.kda_head_dim, c.conv_k
        return (self._view(st.value, (self.B, H, D, D), torch.float32),
                self._view(hi.value, (self.B, 3, H * D, K - 1), torch.float32))

    def mla_cache(self, layer):
        """(latent [B][cap][kv_lora], rope [B][cap][qk_rope]) bf16 bits (int16) views."""
        lt, rp = VP(), VP()
        check(lib.k3gpu_model_mla_cache(self._m, layer, C.byref(lt), C.byref(rp)), "k3gpu_model_mla_cache")
        c = self.lcfg
        lat = self._view(lt.value, (self.B, self.kv_cap, c.kv_lora), torch.int16)
        rope = self._view(rp.value, (self.B, self.kv_cap, c.qk_rope), torch.int16) if rp.value else None
        return lat, rope

    def _view(self, addr, shape, dtype):
        off = addr - self.arena.data_ptr()
        n = 1
        for v in shape:
            n *= v
        nb = n * torch.tensor([], dtype=dtype).element_size()
        return self.arena[off:off + nb].view(dtype).view(*shape)

    def set_ep(self, exchange, shared_banks):
        """Make every layer's MoE step expert parallel over `exchange` (ep.EpExchange): each
        layer's bank must hold this rank's routed experts, shared_banks[L] the replicated
        shared experts of layer L. Every rank must then make the same sweeps."""
        g = exchange.desc
        need = lib.k3gpu_model_ep_workspace(self._m, C.byref(g))
        if need == 0:
            raise K3Error("k3gpu_model_ep_workspace: the exchange does not fit this model")
        self.ep_ws = torch.empty(need + 256, dtype=torch.uint8, device=self.device)
        base = (self.ep_ws.data_ptr() + 255) & ~255
        self._ep_shared = (C.POINTER(K3GpuExpertBank) * len(shared_banks))(
            *[C.pointer(b.desc) for b in shared_banks])
        self._ep_keep = (exchange, shared_banks)
        check(lib.k3gpu_model_set_ep(self._m, C.byref(g), C.cast(self._ep_shared, VP), VP(base), need),
              "k3gpu_model_set_ep")

    def ep_owners_ok(self):
        """The last exchange's per-owner flags (1 = that owner's rows arrived)."""
        world = self._ep_keep[0].world
        ok = (C.c_int * world)()
        check(lib.k3gpu_model_ep_status(self._m, ok), "k3gpu_model_ep_status")
        return list(ok)

    def spec_loop(self, ids, **kw):
        """The engine's decode loop (SpecLoop) with this model's native callbacks (B == 1):
        every verify and commit runs in the library, nothing in Python between them."""
        if self.B != 1:
            raise K3Error("the decode loop drives one sequence")
        return SpecLoop(ids, None, None, native=(lib.k3gpu_model_loop_verify, lib.k3gpu_model_loop_commit,
                                                 self._m), **kw)


def sys_module():
    import sys
    return sys.modules[__name__]
