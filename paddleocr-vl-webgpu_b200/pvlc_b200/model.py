"""End-to-end PaddleOCR-VL greedy OCR on B200: the engine around the attention path.

Architecture (the reference's pinned PaddleOCR-VL-1.6 shapes; random-init fp16 weights):
  * vision encoder: patch projection 3*14*14 -> 1152 (+bias), the learned 27x27
    position table bilinearly interpolated to each image grid
    (crates/pvlc-cpu-ref/src/lib.rs:156-217), 27 pre-LayerNorm layers (eps 1e-6;
    q/k/v/o 1152 with bias; 2-D RoPE; bidirectional attention per image; GELU-tanh
    MLP 4304), post LayerNorm (lib.rs:2880-3064);
  * projector: LayerNorm (eps 1e-5), 2x2 merge to 4608, linear 4608 -> 4608,
    GELU(erf), linear 4608 -> 1024 (lib.rs:2598-2678);
  * decoder: embeddings 103,424 x 1024 with image rows replaced by projector
    outputs (multimodal.rs:115-163), 18 pre-RMSNorm layers (eps 1e-5; q 2048,
    k/v 256, o 2048 -> 1024, no bias; M-RoPE; causal GQA 16/2; SwiGLU 3072),
    final RMSNorm, LM head (lib.rs:1305-1418, 1469-1568), greedy top-1 with EOS 2
    (lib.rs:2201-2305).

Precision: weights and every intermediate activation in fp16; residual streams,
normalisation statistics and logits in f32.  Attention runs on this library's
kernels through the C ABI (vision varlen, decoder causal prefill with the KV
cache written in place -- all prompts of a batch in one launch pair per layer --,
batched split-KV decode with the KV append fused), and so do the elementwise
passes (residual add + LayerNorm / RMSNorm, GELU, SiLU gate; each residual add
rides in the next norm's pass); the dense layers are cuBLAS GEMMs on the same
stream (the vision fc1's GELU in its cuBLASLt epilogue).  The batched decode
step is captured once in a CUDA graph and replayed; tokens are read back once
per chunk of steps, as the reference's chunked greedy driver does
(lib.rs:2309-2366), with the next chunk already queued.

Weight lists are in the canonical order shared with the CPU oracle
(oracle/pvlc_model_oracle.cpp, pvlc_oracle_generate).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import abi, greedy, ops, positions

PROMPT_PREFIX_IDS = (100273, 2969, 93963, 93919, 101305)          # browser_ocr_runtime.mjs:38-40
OCR_PROMPT_SUFFIX_IDS = (101306, 93972, 2497, 93963, 23, 92267, 93963, 23)  # paddleocr_vl_tasks.mjs:4-6


@dataclass(frozen=True)
class ModelConfig:
    vision_layers: int = 27
    vision_hidden: int = 1152
    vision_heads: int = 16
    vision_head_dim: int = 72
    vision_intermediate: int = 4304
    patch_size: int = 14
    channels: int = 3
    pos_side: int = 27
    vision_eps: float = 1e-6
    merge: int = 2
    projector_eps: float = 1e-5
    decoder_layers: int = 18
    hidden: int = 1024
    query_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 128
    intermediate: int = 3072
    vocab: int = 103_424
    rms_eps: float = 1e-5
    eos_token_id: int = 2
    image_token_id: int = positions.IMAGE_TOKEN_ID
    vision_start_token_id: int = positions.VISION_START_TOKEN_ID
    vision_theta: float = positions.VISION_ROPE_THETA
    decoder_theta: float = positions.DECODER_ROPE_THETA

    @property
    def patch_input(self) -> int:
        return self.channels * self.patch_size * self.patch_size

    def oracle_dims(self) -> dict:
        """Field values of the CPU oracle's model-dims struct."""
        return dict(vision_theta=self.vision_theta, decoder_theta=self.decoder_theta,
                    vision_eps=self.vision_eps, projector_eps=self.projector_eps,
                    decoder_eps=self.rms_eps, vision_layers=self.vision_layers,
                    vision_hidden=self.vision_hidden, vision_heads=self.vision_heads,
                    vision_head_dim=self.vision_head_dim,
                    vision_intermediate=self.vision_intermediate, patch_input=self.patch_input,
                    pos_side=self.pos_side, merge=self.merge,
                    decoder_layers=self.decoder_layers, decoder_hidden=self.hidden,
                    query_heads=self.query_heads, kv_heads=self.kv_heads,
                    head_dim=self.head_dim, decoder_intermediate=self.intermediate,
                    vocab=self.vocab, eos_token_id=self.eos_token_id,
                    image_token_id=self.image_token_id,
                    vision_start_token_id=self.vision_start_token_id,
                    sections=positions.MROPE_SECTIONS)


@dataclass
class Weights:
    vision: list
    projector: list
    decoder: list


def init_weights(cfg: ModelConfig, seed: int = 0, device="cuda") -> Weights:
    """Seeded random fp16 weights: linear weights and biases N(0, 0.02^2), norm scales
    1 + N(0, 0.1^2); generated on the device."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def w(*shape, std=0.02):
        return (torch.randn(shape, generator=g, device=device) * std).half()

    def scale(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).half()

    H, I, P = cfg.vision_hidden, cfg.vision_intermediate, cfg.patch_input
    vision = [w(H, P), w(H), w(cfg.pos_side * cfg.pos_side, H)]
    for _ in range(cfg.vision_layers):
        vision += [scale(H), w(H), w(H, H), w(H), w(H, H), w(H), w(H, H), w(H), w(H, H), w(H),
                   scale(H), w(H), w(I, H), w(I), w(H, I), w(H)]
    vision += [scale(H), w(H)]
    M, D = H * cfg.merge * cfg.merge, cfg.hidden
    projector = [scale(H), w(H), w(M, M), w(M), w(D, M), w(D)]
    QW, KW, DI = cfg.query_heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.intermediate
    decoder = [w(cfg.vocab, D)]
    for _ in range(cfg.decoder_layers):
        decoder += [scale(D), w(QW, D), w(KW, D), w(KW, D), w(D, QW), scale(D), w(DI, D),
                    w(DI, D), w(D, DI)]
    decoder += [scale(D), w(cfg.vocab, D)]
    return Weights(vision, projector, decoder)


def ocr_prompt_ids(image_tokens: int, cfg: ModelConfig = ModelConfig()):
    """The engine's OCR prompt: prefix, vision_start, image tokens, task suffix
    (web/engine/browser_ocr_runtime.mjs:38-40,415-421)."""
    return list(PROMPT_PREFIX_IDS) + [cfg.image_token_id] * image_tokens + \
        list(OCR_PROMPT_SUFFIX_IDS)


def _bilinear_axis(source: int, target: int):
    """crates/pvlc-cpu-ref/src/lib.rs:265-278 in f32 for every target index."""
    idx = np.arange(target, dtype=np.float32)
    if target == 1:
        coord = np.zeros(1, np.float32)
    else:
        coord = idx * np.float32(source - 1) / np.float32(target - 1)
    lo = np.minimum(np.floor(coord).astype(np.int64), source - 1)
    hi = np.minimum(lo + 1, source - 1)
    return lo, hi, (coord - lo.astype(np.float32)).astype(np.float32)


class OcrEngine:
    """Batched greedy OCR over images (one image per request)."""

    def __init__(self, cfg: ModelConfig, weights: Weights, device=None,
                 vision_batch_tokens: int = 80_000):
        self.cfg = cfg
        self.device = torch.device(device or "cuda")
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
        self.vision_batch_tokens = vision_batch_tokens
        c = cfg
        vw, pw, dw = weights.vision, weights.projector, weights.decoder
        f32 = lambda t: t.float()   # noqa: E731
        self.patch_w, self.patch_b, self.pos_table = vw[0], vw[1], f32(vw[2])
        self.vlayers = []
        for l in range(c.vision_layers):
            lw = vw[3 + 16 * l: 3 + 16 * (l + 1)]
            # q, k and v as one [3 x 1152, 1152] projection (one GEMM per layer); the
            # attention reads the three column blocks of its output in place
            self.vlayers.append(dict(
                ln1=(f32(lw[0]), f32(lw[1])),
                qkv=(torch.cat([lw[2], lw[4], lw[6]], 0).contiguous(),
                     torch.cat([lw[3], lw[5], lw[7]], 0).contiguous()),
                o=(lw[8], lw[9]), ln2=(f32(lw[10]), f32(lw[11])),
                fc1=(lw[12], lw[13]), fc2=(lw[14], lw[15])))
        post = vw[3 + 16 * c.vision_layers:]
        self.post_ln = (f32(post[0]), f32(post[1]))
        self.proj = dict(ln=(f32(pw[0]), f32(pw[1])), l1=(pw[2], pw[3]), l2=(pw[4], pw[5]))
        self.embed = dw[0]
        self.dlayers = []
        for l in range(c.decoder_layers):
            lw = dw[1 + 9 * l: 1 + 9 * (l + 1)]
            self.dlayers.append(dict(
                n1=f32(lw[0]), q=lw[1], k=lw[2], v=lw[3], o=lw[4], n2=f32(lw[5]),
                qkv=torch.cat([lw[1], lw[2], lw[3]], 0).contiguous(),
                gate_up=torch.cat([lw[6], lw[7]], 0).contiguous(), down=lw[8]))
        self.final_norm = f32(dw[1 + 9 * c.decoder_layers])
        self.lm_head = dw[2 + 9 * c.decoder_layers]
        self._grid_cache = {}
        self._decode = None

    @classmethod
    def from_checkpoint(cls, path, cfg: ModelConfig | None = None, device=None, **kw):
        """Engine over a PaddleOCR-VL-1.6 BF16 safetensors checkpoint: header checked
        against the exact catalog, payload converted to fp16 on the device
        (pvlc_b200.checkpoint.load_weights)."""
        from . import checkpoint
        cfg = cfg or ModelConfig()
        return cls(cfg, checkpoint.load_weights(path, cfg, device), device, **kw)

    # ------------------------------------------------------------- vision side
    def _grid_tables(self, grid):
        """Per-grid device tables: interpolated position embedding (f32), 2-D RoPE, merge order."""
        key = tuple(grid)
        if key in self._grid_cache:
            return self._grid_cache[key]
        t, h, w = key
        S, dev = self.cfg.pos_side, self.device
        y0, y1, yf = _bilinear_axis(S, h)
        x0, x1, xf = _bilinear_axis(S, w)
        tab = self.pos_table
        Y0, X0 = np.meshgrid(y0, x0, indexing="ij")
        Y1, X1 = np.meshgrid(y1, x1, indexing="ij")
        YF, XF = np.meshgrid(yf, xf, indexing="ij")
        gather = lambda yy, xx: tab[torch.from_numpy((yy * S + xx).reshape(-1)).to(dev)]  # noqa
        tl, tr, bl, br = gather(Y0, X0), gather(Y0, X1), gather(Y1, X0), gather(Y1, X1)
        xft = torch.from_numpy(XF.reshape(-1, 1)).to(dev)
        yft = torch.from_numpy(YF.reshape(-1, 1)).to(dev)
        top = tl + (tr - tl) * xft
        bottom = bl + (br - bl) * xft
        pos = (top + (bottom - top) * yft).repeat(t, 1)
        cos, sin = positions.vision_rope_tables([key], self.cfg.vision_head_dim,
                                                self.cfg.vision_theta)
        m = self.cfg.merge
        order = []
        for tt in range(t):
            for my in range(h // m):
                for mx in range(w // m):
                    for py in range(m):
                        for px in range(m):
                            order.append(tt * h * w + (my * m + py) * w + (mx * m + px))
        entry = (pos, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev),
                 torch.tensor(order, dtype=torch.int64, device=dev))
        self._grid_cache[key] = entry
        return entry

    def vision_features(self, patches, grids):
        """patches [N, 588] (f32 or fp16, device) for the images `grids` (pre-merge (t,h,w))
        packed in order -> encoder output [N, 1152] fp16."""
        c = self.cfg
        H, heads, hd = c.vision_hidden, c.vision_heads, c.vision_head_dim
        N = patches.shape[0]
        tabs = [self._grid_tables(g) for g in grids]
        pos = torch.cat([tb[0] for tb in tabs], 0)
        rcos = torch.cat([tb[1] for tb in tabs], 0).contiguous()
        rsin = torch.cat([tb[2] for tb in tabs], 0).contiguous()
        cu = [0]
        for t, h, w in grids:
            cu.append(cu[-1] + t * h * w)
        if cu[-1] != N:
            raise ValueError("patch count does not match the grids")
        x = F.linear(patches.half(), self.patch_w, self.patch_b)
        h32 = x.float() + pos
        ws = torch.empty(ops.vision_workspace_bytes(N, heads, hd), dtype=torch.uint8,
                         device=self.device)
        ctx = torch.empty((N, heads, hd), dtype=torch.float16, device=self.device)
        # each residual add rides in the next norm's pass (ops.add_norm)
        pending = None
        for L in self.vlayers:
            n1 = ops.add_norm(h32, L["ln1"][0], c.vision_eps, bias=L["ln1"][1], delta=pending)
            qkv = F.linear(n1, *L["qkv"])                 # [N, 3 x 1152]
            q, k, v = (qkv[:, j * H:(j + 1) * H].view(N, heads, hd) for j in range(3))
            ops.vision_varlen_attention(q, k, v, cu, rcos, rsin, out=ctx, workspace=ws)
            o = F.linear(ctx.view(N, H), *L["o"])
            n2 = ops.add_norm(h32, L["ln2"][0], c.vision_eps, bias=L["ln2"][1], delta=o)
            # fc1 + bias + GELU-tanh in one cuBLASLt GEMM (GELU epilogue on the f32 result)
            a = torch._addmm_activation(L["fc1"][1], n2, L["fc1"][0].t(), use_gelu=True)
            pending = F.linear(a, *L["fc2"])
        return ops.add_norm(h32, self.post_ln[0], c.vision_eps, bias=self.post_ln[1],
                            delta=pending)

    def project(self, feats, grids):
        """crates/pvlc-cpu-ref/src/lib.rs:2598-2678: [N, 1152] fp16 -> [N/4, 1024] fp16."""
        c = self.cfg
        H, M = c.vision_hidden, c.vision_hidden * c.merge * c.merge
        pre = ops.add_norm(feats.float(), self.proj["ln"][0], c.projector_eps,
                           bias=self.proj["ln"][1])
        order, base = [], 0
        for g in grids:
            order.append(self._grid_tables(g)[3] + base)
            base += g[0] * g[1] * g[2]
        merged = pre.index_select(0, torch.cat(order)).view(-1, M)
        a = ops.gelu_(F.linear(merged, *self.proj["l1"]), erf=True)
        return F.linear(a, *self.proj["l2"])

    def encode_images(self, patches_list, grids, prepare=None):
        """Vision + projector over many images, packed into sub-batches of at most
        vision_batch_tokens patches.  Returns one [tokens_i, 1024] fp16 tensor per image.
        prepare(i, j), when given, queues the work that fills patches_list[i:j] (page
        uploads and the image kernel) just before their sub-batch, so the host's share of
        it overlaps the device's encoding of the previous sub-batch."""
        outs, i = [], 0
        while i < len(grids):
            j, n = i, 0
            while j < len(grids) and (j == i or n + patches_list[j].shape[0] <=
                                      self.vision_batch_tokens):
                n += patches_list[j].shape[0]
                j += 1
            if prepare is not None:
                prepare(i, j)
            p = _join_rows(patches_list[i:j])
            proj = self.project(self.vision_features(p, grids[i:j]), grids[i:j])
            m2 = self.cfg.merge * self.cfg.merge
            outs.extend(torch.split(proj, [g[0] * g[1] * g[2] // m2 for g in grids[i:j]]))
            i = j
        return outs

    # ------------------------------------------------------------ decoder side
    def _prompt_tables(self, ids, grid):
        """M-RoPE tables [3, T, 128] (device) and rope delta of a prompt, cached per
        (prompt, grid): every page of one size shares them."""
        key = (tuple(ids), tuple(grid))
        hit = self._grid_cache.get(key)
        if hit is None:
            c = self.cfg
            pos, delta = positions.mrope_position_ids(ids, [grid])
            pc, ps = positions.mrope_tables(pos, delta, len(ids), c.decoder_theta, c.head_dim)
            hit = (torch.from_numpy(pc).to(self.device), torch.from_numpy(ps).to(self.device),
                   delta)
            self._grid_cache[key] = hit
        return hit

    def _decode_buffers(self, B: int, cap: int) -> "_DecodeGraph":
        """The decode buffers of the last batch shape when (B, cap) matches; otherwise the
        old ones are released first and new ones made."""
        d = self._decode
        if d is None or d.B != B or d.cap != cap:
            self._decode = None
            del d
            torch.cuda.empty_cache()
            self._decode = _DecodeGraph(self, B, cap)
        return self._decode

    def _layer_mlp(self, L, h32, o):
        """h32 += o; SwiGLU MLP of RMSNorm(h32); returns the MLP output (added to h32 by the
        next norm)."""
        c = self.cfg
        n2 = ops.add_norm(h32, L["n2"], c.rms_eps, delta=o)
        return F.linear(ops.silu_mul(F.linear(n2, L["gate_up"])), L["down"])

    def _logits(self, fn):
        return torch.mm(fn, self.lm_head.t(), out_dtype=torch.float32)

    def recognize(self, images, max_new_tokens: int = 512, chunk: int = 32,
                  preprocess_config=None, timings: dict | None = None):
        """Greedy OCR of host RGB8 pages ([H, W, 3] uint8 numpy arrays or CPU tensors).

        Each page is copied to the device (pinned staging), resized and cut into patches
        by the library's image kernel (smart_resize chooses the size), then generate()
        runs the model.  All pages share one device buffer and all patches another, in
        page order, so the call makes two allocations whatever the page count and the
        encoder reads each vision batch's patches in place; each vision batch's pages are
        uploaded and cut just before that batch is encoded.  Returns generate()'s dict."""
        from . import preprocess
        cfgp = preprocess_config or preprocess.MODEL_CONFIG
        ps = cfgp.patch_size
        hosts, sizes = [], []
        for im in images:
            t = im if isinstance(im, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(im))
            if t.dim() != 3 or t.shape[2] != 3 or t.dtype != torch.uint8:
                raise TypeError("pages must be [H, W, 3] uint8")
            if not t.is_pinned():
                t = t.pin_memory()
            H, W = int(t.shape[0]), int(t.shape[1])
            hosts.append(t)
            sizes.append((H, W) + tuple(preprocess.smart_resize(H, W, cfgp)))
        nbytes = [H * W * 3 for H, W, _, _ in sizes]
        npatch = [(h // ps) * (w // ps) for _, _, h, w in sizes]
        rgb = torch.empty(sum(nbytes), dtype=torch.uint8, device=self.device)
        allp = torch.empty((sum(npatch), 3 * ps * ps), dtype=torch.float32, device=self.device)
        ws = torch.empty(max(int(abi.lib().pvlc_image_patches_workspace_bytes(*sz))
                             for sz in sizes), dtype=torch.uint8, device=self.device)
        patches, grids, jobs = [], [], []
        o = r = 0
        for t, (H, W, h, w), nb, n in zip(hosts, sizes, nbytes, npatch):
            patches.append(allp[r:r + n])
            grids.append((1, h // ps, w // ps))
            jobs.append((t, rgb[o:o + nb].view(H, W, 3), h, w))
            o += nb
            r += n

        def prepare(i, j):
            for (t, d, h, w), out in zip(jobs[i:j], patches[i:j]):
                d.copy_(t, non_blocking=True)
                ops.image_patches(d, h, w, ps, out=out, workspace=ws)

        return self.generate(patches, grids, max_new_tokens, chunk=chunk, timings=timings,
                             prepare=prepare)

    def generate(self, images_patches, grids, max_new_tokens: int, chunk: int = 16,
                 record_logits: bool = False, timings: dict | None = None, prepare=None):
        """Greedy OCR of B requests (one image each, same prompt template).

        images_patches: list of [N_i, 588] device tensors; grids: list of (t, h, w).
        Returns dict(tokens=list of lists, stop=list of reasons, logits=optional list of
        [steps_i, vocab] f32 CPU tensors (the logits each token was chosen from)).
        prepare: optional encode_images hook that fills the patches batch by batch.

        Nothing between the first encoder launch and the last decode chunk waits for the
        device except the reads of the first tokens and of each chunk's tokens: the
        prompt plan is built and uploaded (pinned, asynchronous) before the encoder is
        queued, and the next decode chunk is queued before a chunk's tokens are read."""
        c, dev = self.cfg, self.device
        B = len(grids)
        m2 = c.merge * c.merge
        ev = None
        if timings is not None:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            ev[4].record()
        # ---- host-side prompt plan
        ids = [ocr_prompt_ids(g[0] * g[1] * g[2] // m2, c) for g in grids]
        Ts = [len(x) for x in ids]
        cap = max(Ts) + max_new_tokens + 1
        offs = np.concatenate([[0], np.cumsum(Ts)]).astype(np.int64)
        NT = int(offs[-1])
        flat = np.concatenate([np.asarray(x, dtype=np.int64) for x in ids])
        img_pos = np.flatnonzero(flat == c.image_token_id)
        if img_pos.size != sum(g[0] * g[1] * g[2] // m2 for g in grids):
            raise ValueError("image placeholder count does not match the images")
        tables, deltas = [], []
        for x, g in zip(ids, grids):
            tc, ts, delta = self._prompt_tables(x, g)
            tables.append((tc, ts))
            deltas.append(delta)
        plan = _upload(np.concatenate([flat, img_pos, offs[1:] - 1]), dev)
        ids_t, img_idx, last = torch.split(plan, [NT, int(img_pos.size), B])
        if ev:
            ev[0].record()
        img = self.encode_images(images_patches, grids, prepare)
        if ev:
            ev[1].record()
        QW = c.query_heads * c.head_dim
        # the KV caches and the decode step's graph belong to the batch shape (B, cap) and
        # are reused by the next call of the same shape
        dec = self._decode_buffers(B, cap)
        kc, vc = dec.kc, dec.vc
        # ---- prefill: GEMMs over all prompts, attention per prompt
        emb = self.embed.index_select(0, ids_t)
        emb.index_copy_(0, img_idx, torch.cat(img, 0))
        h32 = emb.float()
        ctx = torch.empty((NT, c.query_heads, c.head_dim), dtype=torch.float16, device=dev)
        pending = None
        for l, L in enumerate(self.dlayers):
            n1 = ops.add_norm(h32, L["n1"], c.rms_eps, delta=pending)
            q = F.linear(n1, L["q"]).view(NT, c.query_heads, c.head_dim)
            k = F.linear(n1, L["k"]).view(NT, c.kv_heads, c.head_dim)
            v = F.linear(n1, L["v"]).view(NT, c.kv_heads, c.head_dim)
            ops.decoder_prefill_packed(q, k, v, offs, tables, kc[l], vc[l], ctx)
            pending = self._layer_mlp(L, h32, F.linear(ctx.view(NT, QW), L["o"]))
        fn = ops.add_norm(h32, self.final_norm, c.rms_eps, delta=pending)
        if record_logits:
            logits0 = self._logits(fn.index_select(0, last))
            first = torch.argmax(logits0, dim=-1)
        else:
            first = ops.lm_head_top1(fn.index_select(0, last), self.lm_head).long()
        if ev:
            ev[2].record()
        first_host = _download(first)
        rec = [_download(logits0)] if record_logits else None
        # ---- batched decode, one CUDA graph per step shape; one chunk always queued
        # ahead of the chunk whose tokens are being applied
        dec.reset(first, np.asarray(Ts), np.asarray(deltas))
        inflight = []
        budget = max_new_tokens - 1        # decode steps a request can still need

        def queue(n):
            hist, lg = dec.run(n, record_logits)
            inflight.append((n, _download(hist), _download(lg) if record_logits else None))

        if budget > 0:
            queue(min(chunk, budget))
        first_host[1].synchronize()
        state = greedy.BatchedGreedyState(first_host[0].numpy(), max_new_tokens, c.eos_token_id)
        if record_logits:
            rec[0][1].synchronize()
            rec[0] = rec[0][0]
        while inflight:
            ahead = state.remaining_decode_steps() - sum(x[0] for x in inflight)
            if ahead > 0:
                queue(min(chunk, ahead))
            _, (tok_host, done), lg = inflight.pop(0)
            done.synchronize()
            state.apply_steps(tok_host.numpy())
            if record_logits:
                lg[1].synchronize()
                rec.append(lg[0])
        dec.check_faults()
        if ev:
            ev[3].record()
            ev[3].synchronize()
            timings.update(plan_ms=ev[4].elapsed_time(ev[0]),
                           encode_ms=ev[0].elapsed_time(ev[1]),
                           prefill_ms=ev[1].elapsed_time(ev[2]),
                           decode_ms=ev[2].elapsed_time(ev[3]),
                           decode_steps=int(state.decode_steps.max()))
        out = dict(tokens=[state.generated(b) for b in range(B)],
                   stop=[state.stop_reason(b) for b in range(B)])
        if record_logits:
            allg = torch.cat([r.unsqueeze(0) if r.dim() == 2 else r for r in rec], 0)  # [S,B,V]
            out["logits"] = [allg[: state.count[b], b] for b in range(B)]
        return out


def _join_rows(ts):
    """torch.cat(ts, 0) of [n_i, C] tensors -- as a view, without a copy, when they are
    consecutive row blocks of one buffer (the layout recognize() gives the pages)."""
    first = ts[0]
    if len(ts) == 1:
        return first
    C = first.shape[1]
    expect = first.storage_offset()
    for t in ts:
        if (not t.is_contiguous() or t.dim() != 2 or t.shape[1] != C or t.dtype != first.dtype
                or t.untyped_storage().data_ptr() != first.untyped_storage().data_ptr()
                or t.storage_offset() != expect):
            return torch.cat(ts, 0)
        expect += t.numel()
    return first.as_strided((sum(t.shape[0] for t in ts), C), (C, 1), first.storage_offset())


def _upload(arr, dev):
    """Host array -> device tensor through pinned memory, without waiting for the device."""
    return torch.from_numpy(np.ascontiguousarray(arr)).pin_memory().to(dev, non_blocking=True)


def _download(t):
    """Device tensor -> (pinned host tensor, event): the copy is queued on the current
    stream; the host tensor is valid once the event has completed."""
    host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    host.copy_(t, non_blocking=True)
    done = torch.cuda.Event()
    done.record()
    return host, done


class _DecodeGraph:
    """One batched decode step (embedding -> 18 layers with the fused decode attention ->
    LM head -> argmax), captured in a CUDA graph over static buffers."""

    def __init__(self, eng: OcrEngine, B: int, cap: int):
        """Static buffers of a B-request batch with KV caches of `cap` rows: the caches
        (filled by the prefill), the decode scratch and, once run() first captures it,
        the step graph.  reset() loads a new batch into them."""
        c, dev = eng.cfg, eng.device
        self.eng, self.cap, self.B = eng, cap, B
        Lyr = c.decoder_layers
        self.kc = torch.empty((Lyr, B, cap, c.kv_heads, c.head_dim), dtype=torch.float16,
                              device=dev)
        self.vc = torch.empty_like(self.kc)
        kc, vc = self.kc, self.vc
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.rows = torch.zeros(2 * B, dtype=torch.int32, device=dev)
        self.ct = self.rows[:B]                 # rows before the append
        self.rope_row = self.rows[B:]           # decode position ct + delta
        self.ct_max = 0
        self.rope_rows = 0
        self.rcos = self.rsin = None
        # per-layer device tables of the B cache bases (kc[l, b], vc[l, b])
        Lyr = c.decoder_layers
        lb = np.arange(Lyr * B, dtype=np.int64).reshape(Lyr, B) * (kc.stride(1) * kc.element_size())
        ptrs = _upload(np.concatenate([kc.data_ptr() + lb, vc.data_ptr() + lb], 0), dev)
        self.kp = [ptrs[l] for l in range(Lyr)]
        self.vp = [ptrs[Lyr + l] for l in range(Lyr)]
        self.ws = [ops.DecodeWorkspace(B, dev) for _ in range(Lyr)]
        # one projection GEMM per layer: [B, 2048 | 256 | 256]; decode reads the three
        # column blocks as row-strided views
        QW, KW = c.query_heads * c.head_dim, c.kv_heads * c.head_dim
        self.qkv = torch.empty((B, QW + 2 * KW), dtype=torch.float16, device=dev)
        self.q = self.qkv[:, :QW].view(B, c.query_heads, c.head_dim)
        self.k = self.qkv[:, QW:QW + KW].view(B, c.kv_heads, c.head_dim)
        self.v = self.qkv[:, QW + KW:].view(B, c.kv_heads, c.head_dim)
        self.ctx = torch.empty((B, c.query_heads, c.head_dim), dtype=torch.float16, device=dev)
        # greedy top-1 straight from the LM head GEMM (pvlc_lm_head_top1) unless the
        # caller wants the logits themselves
        self.top1 = torch.empty(B, dtype=torch.int32, device=dev)
        self.top1_ws = torch.empty(
            int(abi.lib().pvlc_lm_head_top1_workspace_bytes(min(B, ops.LM_HEAD_MAX_ROWS))),
            dtype=torch.uint8, device=dev)
        self.graph = None
        self.graph_logits = None
        self.logits = None

    def reset(self, first_tokens, prompt_lens, deltas):
        """A new batch: first tokens (device [B]), host prompt lengths and M-RoPE decode
        deltas [B].  The prefill has written rows [0, prompt_lens[b]) of every cache."""
        c, dev = self.eng.cfg, self.eng.device
        pl = np.asarray(prompt_lens, dtype=np.int64)
        pos = pl + np.asarray(deltas, dtype=np.int64)
        if pos.min() < 0:
            raise positions.PositionError("decode position is negative")
        if len(pl) != self.B or pl.max() >= self.cap:
            raise ValueError("batch does not fit the decode buffers")
        need = int(pos.max()) + self.cap + 1
        if need > self.rope_rows:
            # decode M-RoPE tables (linear positions); the step graph reads them in place
            rc, rs = positions.linear_rope_tables(need, c.decoder_theta, c.head_dim)
            self.rcos, self.rsin = _upload(rc, dev), _upload(rs, dev)
            self.rope_rows = need
            self.graph = None
        self.tok.copy_(first_tokens.to(torch.int64))
        self.rows.copy_(_upload(np.concatenate([pl, pos]).astype(np.int32), dev))
        self.ct_max = int(pl.max())             # host copy of ct.max() (all rows step together)

    def _step(self, with_logits: bool):
        eng, c = self.eng, self.eng.cfg
        B = self.B
        h32 = eng.embed.index_select(0, self.tok).float()
        pending = None
        for l, L in enumerate(eng.dlayers):
            n1 = ops.add_norm(h32, L["n1"], c.rms_eps, delta=pending)
            torch.mm(n1, L["qkv"].t(), out=self.qkv)
            ops.decode(self.q, self.k, self.v, self.rcos, self.rsin, self.kp[l], self.vp[l],
                       self.ct, self.cap, self.cap - 1, self.ws[l], rope_row=self.rope_row,
                       out=self.ctx)
            pending = eng._layer_mlp(L, h32, F.linear(self.ctx.view(B, -1), L["o"]))
        fn = ops.add_norm(h32, eng.final_norm, c.rms_eps, delta=pending)
        if with_logits:
            self.logits = eng._logits(fn)
            self.tok.copy_(torch.argmax(self.logits, dim=-1))
        else:
            ops.lm_head_top1(fn, eng.lm_head, tokens=self.top1, workspace=self.top1_ws)
            self.tok.copy_(self.top1)
        self.rows += 1                          # ct and rope_row advance together

    def _capture(self, with_logits: bool):
        saved = (self.tok.clone(), self.rows.clone())
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step(with_logits)   # warm-up: cuBLAS handles and workspaces
        torch.cuda.current_stream().wait_stream(s)
        # the warm-up wrote cache rows at ct, which the first real step rewrites
        self.tok.copy_(saved[0])
        self.rows.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step(with_logits)
        self.graph_logits = with_logits

    def run(self, steps: int, record_logits: bool = False):
        """Queue `steps` decode steps; returns their [steps, B] tokens (device) and, with
        record_logits, their [steps, B, vocab] logits (device).  Does not wait."""
        if self.ct_max + steps >= self.cap:
            raise abi.PvlcError(abi.CAPACITY_EXHAUSTED, "decode past the cache capacity")
        if self.graph is None or self.graph_logits != record_logits:
            self._capture(record_logits)
        hist = torch.empty((steps, self.B), dtype=torch.int64, device=self.eng.device)
        lg = [] if record_logits else None
        for i in range(steps):
            self.graph.replay()
            hist[i].copy_(self.tok)
            if record_logits:
                lg.append(self.logits.clone())
        self.ct_max += steps
        return hist, (torch.stack(lg, 0) if record_logits else None)

    def check_faults(self):
        """Raise if any decode launch set a device fault flag, or any vision / prefill
        launch ran out of a bounded wait (waits for the device)."""
        flags = sum(w.errors() for w in self.ws)
        if flags:
            raise abi.PvlcError(abi.DEVICE_FAULT_FLAG, f"decode fault flags {flags:#x}")
        kf = ops.fault_flags()
        if kf:
            raise abi.PvlcError(abi.DEVICE_FAULT_FLAG, f"vision / prefill fault flags {kf:#x}")
