"""Device-resident streaming code2wav decoder (``qtts_c2w``).

Packs the decoder weights (named as ``test_stateful_b200.weights.code2wav_param_specs``,
after the module paths of scripts/export/code2wav_streaming.py) into the layouts of
``qtts_c2w_desc`` and drives ``qtts_c2w_step`` — one frame per stream per call,
the way the fused step runs ``Code2WavStreamingWrapper`` at T = 1
(export_09_talker_code2wav_fused.py:145-160).

Packing (all one-time, at load):

* RVQ: each codebook row goes through its ``output_proj`` (a 1x1 conv, linear)
  once, so a frame is a sum of 16 table rows (code2wav_streaming.py:681-706);
  the two projection biases are folded into tables 0 and 1.  fp32.
* Conv ``[out][in][k]`` -> GEMM weight ``[out][k*in]`` (tap-major, matching
  the im2col column order), zero-padded to N % 128 and K % 64.  Where the
  device reads the operand straight from a history buffer (implicit
  convolution: rows per stream a multiple of 128), each tap's channels are
  padded to 64 first, as the buffer's rows are.
* Transposed conv ``[in][out][2s]`` (stride s) -> rows (phase p, out) over
  ``[x(i-1) | x(i)]``: ``W'[p*out+o] = [w[:, o, p+s] | w[:, o, p]]``; the
  upsampling transposed convs (kernel = stride = 2) -> ``W'[p*out+o] = w[:, o, p]``.
* SnakeBeta -> fp32 ``[exp(alpha); exp(-beta)]`` (the exported form,
  code2wav_streaming.py:562-592).
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional

import torch

from .. import _lib
from ..config import Code2WavConfig
from .model import _interleave_gate_up, rope_tables


def _pad_to(t: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    out = torch.zeros(rows, cols, dtype=t.dtype, device=t.device)
    out[:t.shape[0], :t.shape[1]] = t
    return out


def _p64(x):
    return (x + 63) // 64 * 64


def _p128(x):
    return (x + 127) // 128 * 128


def implicit_rows(T: int, max_chunk: int) -> bool:
    """Whether a convolution with T input rows per frame reads the history buffer directly on
    the device (implicit convolution; its weights then pad each tap's channels to 64): when T
    is a multiple of 128, or when the largest call (max_chunk frames) has at least 512 rows per
    stream and pads them to whole 128-row tiles by at most 1/8 (``c2w_implicit_rows`` in
    ``csrc/code2wav.cuh`` applies the same rule)."""
    if T % 128 == 0:
        return True
    rows = max_chunk * T
    pad = -(-rows // 128) * 128 - rows
    return rows >= 512 and pad * 8 <= rows


def pack_code2wav(cfg: Code2WavConfig, W: Dict[str, torch.Tensor], device,
                  max_chunk: int = 1) -> Dict[str, torch.Tensor]:
    """Packed device tensors of the decoder (keys = qtts_c2w_desc field names)."""
    dev = torch.device(device)
    f32 = {k: v.float() for k, v in W.items()}
    bf = lambda t: t.to(device=dev, dtype=torch.bfloat16).contiguous()  # noqa: E731
    fp = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
    P: Dict[str, object] = {}
    # ---- RVQ tables through output_proj
    wf = f32["c2w.rvq_first.output_proj.weight"][:, :, 0]
    wr = f32["c2w.rvq_rest.output_proj.weight"][:, :, 0]
    tabs = [f32["c2w.rvq_first.codebook.0"] @ wf.t() + f32["c2w.rvq_first.output_proj.bias"]]
    for g in range(cfg.num_codebooks - 1):
        t = f32[f"c2w.rvq_rest.codebook.{g}"] @ wr.t()
        if g == 0:
            t = t + f32["c2w.rvq_rest.output_proj.bias"]
        tabs.append(t)
    P["rvq_tables"] = fp(torch.stack(tabs))

    def conv_w(name, n_pad=None, k_pad=None, in_pad=None):
        """[out, in, k] -> [out, k * in_pad] (tap-major, each tap's channels padded to in_pad)."""
        w = f32[name]  # [out, in, k]
        o, i, k = w.shape
        ip = in_pad or i
        m = torch.zeros(o, k, ip)
        m[:, :, :i] = w.permute(0, 2, 1)
        m = m.reshape(o, k * ip)
        return bf(_pad_to(m, n_pad or _p128(o), k_pad or _p64(k * ip)))

    # implicit-convolution blocks (see implicit_rows) pad each tap's channels to 64
    T, t_in, t_blk = 4, [], []
    for r_ in cfg.upsample_rates:
        t_in.append(T)
        T *= r_
        t_blk.append(T)

    def vec(name, n_pad=None):
        v = f32[name]
        out = torch.zeros(n_pad or v.numel())
        out[:v.numel()] = v
        return bf(out)

    def snake(pa, pb):
        return fp(torch.stack([torch.exp(f32[pa]), torch.exp(-f32[pb])]))

    P["w_pre_conv"] = conv_w("c2w.pre_conv.weight", cfg.latent_dim)
    P["b_pre_conv"] = vec("c2w.pre_conv.bias")
    p = "c2w.pre_transformer."
    P["w_in_proj"] = bf(f32[p + "input_proj.weight"])
    P["b_in_proj"] = vec(p + "input_proj.bias")
    L = cfg.num_layers
    lay = lambda n: [f32[f"{p}layers.{i}.{n}"] for i in range(L)]  # noqa: E731
    P["w_in_norm"] = bf(torch.stack(lay("input_layernorm.weight")))
    P["w_qkv"] = bf(torch.stack([torch.cat([q, k, v]) for q, k, v in zip(
        lay("self_attn.q_proj.weight"), lay("self_attn.k_proj.weight"), lay("self_attn.v_proj.weight"))]))
    P["w_q_norm"] = bf(torch.stack(lay("self_attn.q_norm.weight")))
    P["w_k_norm"] = bf(torch.stack(lay("self_attn.k_norm.weight")))
    P["w_o"] = bf(torch.stack(lay("self_attn.o_proj.weight")))
    P["attn_scale"] = bf(torch.stack(lay("self_attn_layer_scale.scale")))
    P["w_post_norm"] = bf(torch.stack(lay("post_attention_layernorm.weight")))
    P["w_gate_up"] = bf(torch.stack([_interleave_gate_up(g, u) for g, u in zip(
        lay("mlp.gate_proj.weight"), lay("mlp.up_proj.weight"))]))
    P["w_down"] = bf(torch.stack(lay("mlp.down_proj.weight")))
    P["mlp_scale"] = bf(torch.stack(lay("mlp_layer_scale.scale")))
    P["w_final_norm"] = bf(f32[p + "norm.weight"])
    P["w_out_proj"] = bf(f32[p + "output_proj.weight"])
    P["b_out_proj"] = vec(p + "output_proj.bias")
    LAT = cfg.latent_dim
    for i in range(2):
        u = f"c2w.upsample.{i}."
        w = f32[u + "transconv.weight"]  # [in, out, 2]
        P[f"up_w{i}"] = bf(torch.cat([w[:, :, 0].t(), w[:, :, 1].t()]))
        P[f"up_b{i}"] = bf(f32[u + "transconv.bias"].repeat(2))
        P[f"dw_w{i}"] = fp(f32[u + "convnext.dwconv.weight"][:, 0, :])
        P[f"dw_b{i}"] = fp(f32[u + "convnext.dwconv.bias"])
        P[f"ln_w{i}"] = fp(f32[u + "convnext.norm.weight"])
        P[f"ln_b{i}"] = fp(f32[u + "convnext.norm.bias"])
        P[f"pw1_w{i}"] = bf(f32[u + "convnext.pwconv1.weight"])
        P[f"pw1_b{i}"] = vec(u + "convnext.pwconv1.bias")
        P[f"pw2_w{i}"] = bf(f32[u + "convnext.pwconv2.weight"])
        P[f"pw2_b{i}"] = vec(u + "convnext.pwconv2.bias")
        P[f"gamma{i}"] = vec(u + "convnext.gamma")
    P["w_conv0"] = conv_w("c2w.decoder.0.weight")
    P["b_conv0"] = vec("c2w.decoder.0.bias", _p128(cfg.decoder_dim))
    for b, (cin, cout, s) in enumerate(cfg.block_dims()):
        k = f"c2w.decoder.{1 + b}."
        P[f"blk_snake{b}"] = snake(k + "snake.alpha", k + "snake.beta")
        w = f32[k + "transconv.weight"]  # [cin, cout, 2s]
        cinp = _p64(cin) if implicit_rows(t_in[b], max_chunk) else cin
        rows = []
        for ph in range(s):
            r2 = torch.zeros(cout, 2, cinp)
            r2[:, 0, :cin] = w[:, :, ph + s].t()  # tap x(i-1)
            r2[:, 1, :cin] = w[:, :, ph].t()      # tap x(i)
            rows.append(r2.reshape(cout, 2 * cinp))
        P[f"blk_tw{b}"] = bf(_pad_to(torch.cat(rows), _p128(s * cout), _p64(2 * cinp)))
        coutp = _p64(cout) if implicit_rows(t_blk[b], max_chunk) else cout
        bias = torch.zeros(_p128(s * cout))
        bias[:s * cout] = f32[k + "transconv.bias"].repeat(s)
        P[f"blk_tb{b}"] = bf(bias)
        for j, _ in enumerate(cfg.dilations):
            r = f"{k}res.{j}."
            P[f"res_act1_{b}_{j}"] = snake(r + "act1.alpha", r + "act1.beta")
            P[f"res_act2_{b}_{j}"] = snake(r + "act2.alpha", r + "act2.beta")
            P[f"res_w1_{b}_{j}"] = conv_w(r + "conv1.weight", in_pad=coutp)
            P[f"res_b1_{b}_{j}"] = vec(r + "conv1.bias", _p128(cout))
            P[f"res_w2_{b}_{j}"] = conv_w(r + "conv2.weight", _p128(cout), _p128(cout))
            P[f"res_b2_{b}_{j}"] = vec(r + "conv2.bias", _p128(cout))
    P["final_snake"] = snake("c2w.decoder.5.alpha", "c2w.decoder.5.beta")
    P["final_w"] = fp(f32["c2w.decoder.6.weight"][0].t())  # [7][C]
    P["final_b"] = float(f32["c2w.decoder.6.bias"][0])
    return P


_STATE_DTYPES = {0: torch.bfloat16, 1: torch.float32, 2: torch.float16}


def expected_state_layout(cfg: Code2WavConfig, max_chunk: int = 1):
    """The decoder's state parts (``qtts_c2w_state_layout``) computed on the host: the window
    KV, then the causal convolutions' contexts (pre_conv, the two ConvNeXt depthwise inputs in
    fp32, conv k7, 4 blocks x 3 residual units, the last conv) and the 4 transposed convs'
    previous input rows; implicit-convolution buffers pad their channels to 64."""
    parts = [(cfg.num_layers * 2 * cfg.num_heads * cfg.window, cfg.head_dim, cfg.head_dim, 2)]
    parts.append((2, cfg.codebook_dim, cfg.codebook_dim, 0))
    parts += [(6, cfg.latent_dim, cfg.latent_dim, 1)] * 2
    parts.append((6, cfg.latent_dim, cfg.latent_dim, 0))
    T, t_in, t_blk = 4, [], []
    for r_ in cfg.upsample_rates:
        t_in.append(T)
        T *= r_
        t_blk.append(T)
    dims = cfg.block_dims()
    for b, (cin, cout, _) in enumerate(dims):
        cp = _p64(cout) if implicit_rows(t_blk[b], max_chunk) else cout
        parts += [(6 * d, cp, cout, 0) for d in cfg.dilations]
    parts.append((6, dims[-1][1], dims[-1][1], 0))
    for b, (cin, _, _) in enumerate(dims):
        parts.append((1, _p64(cin) if implicit_rows(t_in[b], max_chunk) else cin, cin, 0))
    return parts


def warm_state_parts(cfg: Code2WavConfig, packed: Dict[str, torch.Tensor], layout, c2w_kv, conv_states,
                     transconv_states, frame_idx: int, device, tail_qr: Optional[dict] = None) -> List[torch.Tensor]:
    """A warm decoder state in the reference's layout (``Executor.apply_c2w_warm_state``,
    engine/backend/executor.py:715-757) as this decoder's state parts (``qtts_c2w_state_part``).

    * ``c2w_kv`` [1, 2 * layers, heads, T, head_dim] (k, v of layer l at 2l, 2l + 1; keys
      RoPE-rotated at their absolute frame): cropped to window - 1 past frames as the reference
      does, frame ``frame_idx - T + i`` written at window position ``(frame_idx - T + i) % window``.
    * ``conv_states[j]`` [1, channels, ctx] (the activated conv inputs,
      code2wav_streaming.py:73-93): transposed to rows, channels zero-padded to the row.
    * ``transconv_states[b]`` [1, C_out, s]: the reference keeps the bias-free overlap tail
      ``tail[c, p] = sum_i W[i, c, s + p] x_prev[i]`` (code2wav_streaming.py:96-126); this
      decoder keeps ``x_prev`` itself.  With C_out * s >= C_in the map is injective for a
      full-rank W, so ``x_prev`` is its least-squares solution, using the packed x(i-1) tap of
      the block's transposed-conv weights (rows (phase, out channel)).

    The conversion runs on the host (float64 QR of each tap, cached in ``tail_qr`` per block)
    and the parts are moved to ``device`` at the end.  Raises ``ValueError`` on any shape that
    does not match this decoder."""
    out_dev = torch.device(device)
    dev = torch.device("cpu")
    parts: List[torch.Tensor] = []
    L, H, D, Wn = cfg.num_layers, cfg.num_heads, cfg.head_dim, cfg.window
    kv = torch.as_tensor(c2w_kv).to(dev, torch.float32)
    if kv.dim() == 5:
        if kv.shape[0] != 1:
            raise ValueError(f"c2w_kv batch {kv.shape[0]} != 1")
        kv = kv[0]
    if kv.dim() != 4 or tuple(kv.shape[:2]) != (2 * L, H) or kv.shape[3] != D:
        raise ValueError(f"c2w_kv shape {tuple(kv.shape)} does not match [2*{L}, {H}, T, {D}]")
    kv = kv[:, :, -max(1, Wn - 1):, :]
    T = kv.shape[2]
    ring = torch.zeros(2 * L, H, Wn, D, device=dev, dtype=torch.float32)
    pos = (torch.arange(T, device=dev) + (int(frame_idx) - T)) % Wn
    ring[:, :, pos, :] = kv
    parts.append(ring.reshape(-1, D).to(torch.float16).contiguous())
    if len(conv_states) != len(layout) - 1 - 4 or len(transconv_states) != 4:
        raise ValueError(f"{len(conv_states)} conv / {len(transconv_states)} transconv states, expected "
                         f"{len(layout) - 5} / 4")
    for j, st in enumerate(conv_states):
        rows, row_elems, valid, dt = layout[1 + j]
        t = torch.as_tensor(st).to(dev, torch.float32)
        t = t.reshape(t.shape[-2], t.shape[-1])  # [channels, ctx]
        if tuple(t.shape) != (valid, rows):
            raise ValueError(f"conv_state_{j} shape {tuple(t.shape)} != [{valid}, {rows}]")
        part = torch.zeros(rows, row_elems, device=dev, dtype=torch.float32)
        part[:, :valid] = t.t()
        parts.append(part.to(_STATE_DTYPES[dt]).contiguous())
    for b, (st, (cin, cout, s)) in enumerate(zip(transconv_states, cfg.block_dims())):
        rows, row_elems, valid, dt = layout[1 + len(conv_states) + b]
        tail = torch.as_tensor(st).to(dev, torch.float32)
        tail = tail.reshape(tail.shape[-2], tail.shape[-1])  # [C_out, s]
        if tuple(tail.shape) != (cout, s) or valid != cin or rows != 1:
            raise ValueError(f"transconv_overlap_{b} shape {tuple(tail.shape)} != [{cout}, {s}]")
        qr = tail_qr.get(b) if tail_qr is not None else None
        if qr is None:  # tap x(i-1), rows (phase, c): A = Q R
            A = packed[f"blk_tw{b}"][: s * cout, :cin].to("cpu", torch.float64)
            qr = torch.linalg.qr(A)
            if tail_qr is not None:
                tail_qr[b] = qr
        Q, R = qr
        rhs = tail.t().reshape(-1, 1).to(torch.float64)
        x_prev = torch.linalg.solve_triangular(R, Q.t() @ rhs, upper=True)[:, 0]
        part = torch.zeros(1, row_elems, device=dev, dtype=torch.float32)
        part[0, :cin] = x_prev.to(torch.float32)
        parts.append(part.to(_STATE_DTYPES[dt]).contiguous())
    return [t.to(out_dev).contiguous() for t in parts]


class DeviceCode2Wav:
    """Packed weights + native decoder state for ``max_slots`` streams on one GPU."""

    def __init__(self, cfg: Code2WavConfig, weights: Dict[str, torch.Tensor], device, max_slots: int,
                 max_frames: int = 4096, max_chunk: int = 1):
        self.cfg = cfg
        self.device = torch.device(device)
        self.max_slots = max_slots
        self.samples_per_frame = cfg.samples_per_frame
        self.P = pack_code2wav(cfg, weights, self.device, max_chunk=max_chunk)
        self.rope_cos, self.rope_sin = rope_tables(cfg.head_dim, cfg.rope_theta, max_frames, self.device)
        P = self.P
        d = _lib.C2wDesc()
        d.num_codebooks, d.codebook_size, d.codebook_dim = cfg.num_codebooks, cfg.codebook_size, cfg.codebook_dim
        d.latent, d.hidden, d.layers = cfg.latent_dim, cfg.hidden_size, cfg.num_layers
        d.heads, d.head_dim, d.inter = cfg.num_heads, cfg.head_dim, cfg.intermediate_size
        d.window, d.decoder_dim = cfg.window, cfg.decoder_dim
        d.convnext_dim = cfg.convnext_mult * cfg.latent_dim
        d.max_slots, d.max_frames, d.max_chunk = max_slots, max_frames, max_chunk
        self.max_chunk = max_chunk
        d.up_ratio[:] = list(cfg.upsample_ratios)
        d.rates[:] = list(cfg.upsample_rates)
        d.dilations[:] = list(cfg.dilations)
        d.rms_eps, d.ln_eps = cfg.rms_eps, cfg.ln_eps
        for name in ("rvq_tables", "w_pre_conv", "b_pre_conv", "w_in_proj", "b_in_proj", "w_in_norm", "w_qkv",
                     "w_q_norm", "w_k_norm", "w_o", "attn_scale", "w_post_norm", "w_gate_up", "w_down", "mlp_scale",
                     "w_final_norm", "w_out_proj", "b_out_proj", "w_conv0", "b_conv0", "final_snake", "final_w"):
            setattr(d, name, P[name].data_ptr())
        d.rope_cos, d.rope_sin = self.rope_cos.data_ptr(), self.rope_sin.data_ptr()
        for i in range(2):
            for f in ("up_w", "up_b", "dw_w", "dw_b", "ln_w", "ln_b", "pw1_w", "pw1_b", "pw2_w", "pw2_b", "gamma"):
                getattr(d, f)[i] = P[f"{f}{i}"].data_ptr()
        for b in range(4):
            d.blk_snake[b] = P[f"blk_snake{b}"].data_ptr()
            d.blk_tw[b] = P[f"blk_tw{b}"].data_ptr()
            d.blk_tb[b] = P[f"blk_tb{b}"].data_ptr()
            for j in range(3):
                for f in ("res_act1", "res_act2", "res_w1", "res_b1", "res_w2", "res_b2"):
                    getattr(d, f)[b][j] = P[f"{f}_{b}_{j}"].data_ptr()
        d.final_b = P["final_b"]
        self.desc = d
        lib = _lib.load()
        h = C.c_void_p()
        torch.cuda.synchronize(self.device)
        _lib.check(lib.qtts_c2w_create(C.byref(d), C.byref(h)), "c2w_create")
        self.handle = h
        self.last_launches = 0
        self.tail_qr: dict = {}  # warm-state conversion: QR of each block's x(i-1) tap (host, float64)

    def set_background(self, on: bool = True) -> None:
        """Mark the decoder as running beside a latency-critical stream (its kernels then launch
        without programmatic dependent launch; see ``qtts_c2w_set_background``)."""
        _lib.check(_lib.load().qtts_c2w_set_background(self.handle, int(bool(on))), "c2w_set_background")

    def reset(self, slots: torch.Tensor, stream=None) -> None:
        """Start new streams (frame 0, zero conv/transconv state) on ``slots`` (device int32)."""
        lib = _lib.load()
        _lib.check(lib.qtts_c2w_reset(self.handle, _lib.ptr(slots), int(slots.numel()), _lib.stream_ptr(stream)),
                   "c2w_reset")

    def step(self, codes: torch.Tensor, slots: torch.Tensor, wav: torch.Tensor, n: int = None, stream=None,
             frames: int = 1) -> None:
        """``frames`` frames per stream: ``codes`` int64 [n][>=16] (frames = 1) or [n][frames][16]
        (device, contiguous), ``slots`` int32 [n], ``wav`` fp32 [n][frames * 1920]."""
        n = int(slots.numel()) if n is None else n
        assert codes.dtype == torch.int64 and slots.dtype == torch.int32 and wav.dtype == torch.float32
        ld = int(codes.stride(-2)) if codes.dim() == 3 else int(codes.stride(0))
        if codes.dim() == 3:
            assert codes.is_contiguous() and codes.shape[1] == frames
        lib = _lib.load()
        _lib.check(lib.qtts_c2w_step(self.handle, _lib.ptr(codes), ld, frames, _lib.ptr(slots), n,
                                     _lib.ptr(wav), _lib.stream_ptr(stream)), "c2w_step")
        self.last_launches = lib.qtts_c2w_launches(self.handle)

    def state_layout(self):
        """[(rows, row_elems, valid_elems, dtype)] of the 22 state parts (``qtts_c2w_state_layout``)."""
        parts = (_lib.C2wStatePart * _lib.C2W_STATE_PARTS)()
        _lib.check(_lib.load().qtts_c2w_state_layout(self.handle, parts, _lib.C2W_STATE_PARTS), "c2w_state_layout")
        return [(p.rows, p.row_elems, p.valid_elems, p.dtype) for p in parts]

    def install_state(self, slot: int, parts: List[torch.Tensor], frame: int, stream=None) -> None:
        """Write a slot's state parts (``warm_state_parts``) and set its frame counter, ordered on
        ``stream``."""
        lib = _lib.load()
        layout = self.state_layout()
        if len(parts) != len(layout):
            raise ValueError(f"{len(parts)} state parts, the decoder has {len(layout)}")
        for i, (t, (rows, row_elems, _, dt)) in enumerate(zip(parts, layout)):
            if (tuple(t.shape) != (rows, row_elems) or t.dtype != _STATE_DTYPES[dt] or not t.is_contiguous()
                    or t.device != self.device):
                raise ValueError(f"state part {i}: {tuple(t.shape)} {t.dtype} != ({rows}, {row_elems}) "
                                 f"{_STATE_DTYPES[dt]} on {self.device}")
            _lib.check(lib.qtts_c2w_write_state(self.handle, int(slot), i, t.data_ptr(), t.numel() * t.element_size(),
                                                _lib.stream_ptr(stream)), "c2w_write_state")
        _lib.check(lib.qtts_c2w_set_frame(self.handle, int(slot), int(frame), _lib.stream_ptr(stream)),
                   "c2w_set_frame")

    def close(self) -> None:
        if self.handle:
            _lib.load().qtts_c2w_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
