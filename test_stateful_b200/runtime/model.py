"""Device-resident model, paged KV pool and engine handle.

Weights arrive with the reference's module names (``test_stateful_b200.weights``)
and are packed once into the layouts the kernels stream:

* ``w_qkv``     [L][(Hq+2Hkv)·D][H]  — q_proj, k_proj, v_proj rows stacked
  (talker_unified_modules.py:173-175), so one GEMM and one epilogue produce q,
  k and v;
* ``w_gate_up`` [L][2I][H]           — gate/up rows interleaved in 64-row groups
  (tile t = gate[64t:64t+64] then up[64t:64t+64]) so the SwiGLU epilogue finds
  both halves of a feature in one 128-row tile (Qwen3MLP);
* ``w_o``, ``w_down``, norms          — stacked per layer.

The paged KV pool is ``[num_blocks][L][2][Hkv][16][D]`` fp16: one block of one
(layer, k|v, head) is a contiguous 4 KB chunk, the unit the attention kernel
copies into shared memory; a whole block (all layers) is one contiguous
region, the unit of a copy-on-write.
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, Optional

import torch

from .. import _lib
from ..config import EngineConfig


def rope_tables(head_dim: int, theta: float, max_pos: int, device) -> tuple:
    """cos/sin ``[max_pos, D/2]`` fp32: ``freqs = pos * inv_freq`` in fp32 as
    talker_unified_modules.py:92-107 computes them (``attention_scaling`` = 1)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float32).unsqueeze(1)
    freqs = pos * inv_freq.unsqueeze(0)
    return freqs.cos().contiguous().to(device), freqs.sin().contiguous().to(device)


def _interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    I, H = gate.shape
    g = gate.view(I // 64, 64, H)
    u = up.view(I // 64, 64, H)
    return torch.stack([g, u], dim=1).reshape(2 * I, H)


class PagedPoolTensors:
    """Device arrays of the paged allocator plus the KV block storage."""

    def __init__(self, cfg: EngineConfig, device):
        t, p = cfg.talker, cfg.pool
        i32 = dict(device=device, dtype=torch.int32)
        self.free_stack = torch.empty(p.num_blocks, **i32)
        self.free_top = torch.empty(1, **i32)
        self.refcount = torch.empty(p.num_blocks, **i32)
        self.block_table = torch.empty(p.max_slots, p.max_blocks_per_seq, **i32)
        self.seq_len = torch.empty(p.max_slots, **i32)
        self.position_offset = torch.empty(p.max_slots, **i32)
        # zero-filled: attention kernels multiply V rows past a sequence's last key by P = 0, so the
        # pool must never hold a non-finite value (it only ever receives written K/V after this)
        self.kv = torch.zeros(p.num_blocks, t.num_layers, 2, t.kv_heads, p.block_size, t.head_dim,
                              device=device, dtype=torch.float16)
        self.block_elems = t.num_layers * 2 * t.kv_heads * p.block_size * t.head_dim
        self.state = _lib.PagedState(
            self.free_stack.data_ptr(), self.free_top.data_ptr(), self.refcount.data_ptr(),
            self.block_table.data_ptr(), self.seq_len.data_ptr(), self.position_offset.data_ptr(),
            p.num_blocks, p.block_size, p.max_slots, p.max_blocks_per_seq)

    def init(self, stream=None):
        lib = _lib.load()
        _lib.check(lib.qtts_sched_init(C.byref(self.state), _lib.stream_ptr(stream)), "sched_init")


class DeviceModel:
    """Packed weights + pool + native engine for one GPU."""

    def __init__(self, cfg: EngineConfig, weights: Dict[str, torch.Tensor], device, max_batch: int,
                 max_prefill_rows: int = 512):
        self.cfg = cfg
        self.device = torch.device(device)
        self.max_batch = max_batch
        self.max_prefill_rows = max_prefill_rows
        t, c = cfg.talker, cfg.cp
        dev = self.device
        bf = torch.bfloat16

        def w(name):
            return weights[name].to(device=dev, dtype=bf)

        L, H, I = t.num_layers, t.hidden_size, t.intermediate_size
        qkv_rows = t.q_size + 2 * t.kv_size
        self.w_qkv = torch.empty(L, qkv_rows, H, device=dev, dtype=bf)
        self.w_o = torch.empty(L, H, t.q_size, device=dev, dtype=bf)
        self.w_gate_up = torch.empty(L, 2 * I, H, device=dev, dtype=bf)
        self.w_down = torch.empty(L, H, I, device=dev, dtype=bf)
        self.w_in_norm = torch.empty(L, H, device=dev, dtype=bf)
        self.w_post_norm = torch.empty(L, H, device=dev, dtype=bf)
        self.w_q_norm = torch.empty(L, t.head_dim, device=dev, dtype=bf)
        self.w_k_norm = torch.empty(L, t.head_dim, device=dev, dtype=bf)
        for l in range(L):
            p = f"talker.layers.{l}."
            self.w_qkv[l] = torch.cat([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                                       w(p + "self_attn.v_proj.weight")], 0)
            self.w_o[l] = w(p + "self_attn.o_proj.weight")
            self.w_gate_up[l] = _interleave_gate_up(w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight"))
            self.w_down[l] = w(p + "mlp.down_proj.weight")
            self.w_in_norm[l] = w(p + "input_layernorm.weight")
            self.w_post_norm[l] = w(p + "post_attention_layernorm.weight")
            self.w_q_norm[l] = w(p + "self_attn.q_norm.weight")
            self.w_k_norm[l] = w(p + "self_attn.k_norm.weight")
        self.w_final_norm = w("talker.norm.weight")
        self.w_codec_head = w("talker.codec_head.weight")
        self.w_codec_emb = w("talker.codec_embedding.weight")
        self.max_pos = cfg.pool.max_seq_len + 64
        self.rope_cos, self.rope_sin = rope_tables(t.head_dim, t.rope_theta, self.max_pos, dev)

        CL, CH, CI = c.num_layers, c.hidden_size, c.intermediate_size
        cqkv = (c.num_heads + 2 * c.kv_heads) * c.head_dim
        self.cp_w_proj = w("cp.projection.weight")
        self.cp_b_proj = w("cp.projection.bias")
        self.cp_w_qkv = torch.empty(CL, cqkv, CH, device=dev, dtype=bf)
        self.cp_w_o = torch.empty(CL, CH, c.num_heads * c.head_dim, device=dev, dtype=bf)
        self.cp_w_gate_up = torch.empty(CL, 2 * CI, CH, device=dev, dtype=bf)
        self.cp_w_down = torch.empty(CL, CH, CI, device=dev, dtype=bf)
        self.cp_w_in_norm = torch.empty(CL, CH, device=dev, dtype=bf)
        self.cp_w_post_norm = torch.empty(CL, CH, device=dev, dtype=bf)
        self.cp_w_q_norm = torch.empty(CL, c.head_dim, device=dev, dtype=bf)
        self.cp_w_k_norm = torch.empty(CL, c.head_dim, device=dev, dtype=bf)
        for l in range(CL):
            p = f"cp.layers.{l}."
            self.cp_w_qkv[l] = torch.cat([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                                          w(p + "self_attn.v_proj.weight")], 0)
            self.cp_w_o[l] = w(p + "self_attn.o_proj.weight")
            self.cp_w_gate_up[l] = _interleave_gate_up(w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight"))
            self.cp_w_down[l] = w(p + "mlp.down_proj.weight")
            self.cp_w_in_norm[l] = w(p + "input_layernorm.weight")
            self.cp_w_post_norm[l] = w(p + "post_attention_layernorm.weight")
            self.cp_w_q_norm[l] = w(p + "self_attn.q_norm.weight")
            self.cp_w_k_norm[l] = w(p + "self_attn.k_norm.weight")
        self.cp_w_final_norm = w("cp.norm.weight")
        self.cp_w_lm_head = torch.stack([w(f"cp.lm_head.{s}.weight") for s in range(c.num_stages)])
        self.cp_w_codec_emb = torch.stack([w(f"cp.codec_embedding.{s}.weight") for s in range(c.num_stages)])
        self.cp_rope_cos, self.cp_rope_sin = rope_tables(c.head_dim, c.rope_theta, c.num_stages + 1, dev)

        self.pool = PagedPoolTensors(cfg, dev)
        self.pool.init()
        self.engine = C.c_void_p()
        self._create_engine()

    # ------------------------------------------------------------------
    def _create_engine(self):
        t, c = self.cfg.talker, self.cfg.cp
        d = _lib.ModelDesc()
        d.layers, d.hidden, d.heads, d.kv_heads = t.num_layers, t.hidden_size, t.num_heads, t.kv_heads
        d.head_dim, d.inter, d.vocab, d.eos_id, d.topk = (t.head_dim, t.intermediate_size, t.codec_vocab_size,
                                                          t.codec_eos_id, t.logits_topk)
        d.rms_eps = t.rms_eps
        for name in ("w_qkv", "w_o", "w_gate_up", "w_down", "w_in_norm", "w_post_norm", "w_q_norm", "w_k_norm",
                     "w_final_norm", "w_codec_head", "w_codec_emb", "rope_cos", "rope_sin",
                     "cp_w_proj", "cp_b_proj", "cp_w_qkv", "cp_w_o", "cp_w_gate_up", "cp_w_down", "cp_w_in_norm",
                     "cp_w_post_norm", "cp_w_q_norm", "cp_w_k_norm", "cp_w_final_norm", "cp_w_lm_head",
                     "cp_w_codec_emb", "cp_rope_cos", "cp_rope_sin"):
            setattr(d, name, getattr(self, name).data_ptr())
        d.max_pos = self.max_pos
        d.cp_layers, d.cp_hidden, d.cp_heads, d.cp_kv_heads = c.num_layers, c.hidden_size, c.num_heads, c.kv_heads
        d.cp_head_dim, d.cp_inter, d.cp_vocab, d.cp_stages = c.head_dim, c.intermediate_size, c.vocab_size, c.num_stages
        d.cp_rms_eps = c.rms_eps
        d.pool = self.pool.state
        d.kv_pool = self.pool.kv.data_ptr()
        d.max_batch = self.max_batch
        d.max_prefill_rows = self.max_prefill_rows
        self._desc = d
        torch.cuda.synchronize(self.device)
        _lib.check(_lib.load().qtts_engine_create(C.byref(d), C.byref(self.engine)), "engine_create")

    def step(self, io: _lib.StepIO, stream=None) -> None:
        _lib.check(_lib.load().qtts_engine_step(self.engine, C.byref(io), _lib.stream_ptr(stream)), "engine_step")

    def close(self) -> None:
        if self.engine:
            torch.cuda.synchronize(self.device)
            _lib.load().qtts_engine_destroy(self.engine)
            self.engine = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
