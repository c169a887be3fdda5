"""The reference's 128-dim model trained step by step, written twice: once on
the oracle (CPU restatements of the path's operators plus numpy for the
rest of the model) and once on this library's CUDA kernels through the C ABI
(torch on the device for the parts outside the path).  Test infrastructure:
the tests compare the two loss curves.

What both arms follow, from the reference:

- model: ModelConfig::default_128 (src/model.rs:26-35): 64 bands (n_embd
  128), 4 heads, 4 blocks, maestro_dim 16, block_size 256, rk4_n_steps 8;
- initialisation: init_model_ext with seed 42 (src/init.rs:96-144) drawing
  every trainable weight from the xorshift64 generator of src/rng.rs:5-45 in
  the reference's order (block 0: c_attn, c_proj, PerBandLinear band_w then
  out_proj; blocks 1-3: c_attn, c_proj, maestro squeeze, process_1,
  out_proj; then lm_head), LayerNorm 1 / 0, KerrWeights gamma_raw =
  softplus^-1(0.1), omega_k = (k+1)/64, alpha = beta = 0.1;
- frozen embeddings: the harmonic token table and the positional table
  (src/model.rs:104-135);
- forward: src/pipeline.rs:177-360 (curriculum band masking of the
  embedding, LN1 / attention / residual / LN2 / FFN / residual per block,
  ln_f, lm_head without bias); FFN of block 0 is PerBandLinear
  (src/backend.rs:483-505), of blocks 1-3 KerrMaestroAdd
  (src/backend.rs:537-553: Kerr-ODE + maestro (squeeze, GELU, process_1),
  then out_proj);
- loss and backward: per-position cross-entropy averaged over the sequence
  (src/pipeline.rs:364-422), the FFN and attention backward of
  src/pipeline.rs:427-758 and src/backward.rs (GELU :132-147, cross-entropy
  :159-170);
- step: gradients summed over the batch and divided by batch_size, global
  norm clipped to 1.0, Adam (0.9, 0.999, eps 1e-8, bias correction) at lr
  3e-4 (src/train.rs:231-277, src/optim.rs:9-83, src/main.rs:486-490);
- curriculum: default_3stage over the reference's default 3000 iterations
  (src/train.rs:27-69), so the first steps run with 8 active bands;
- data: a seeded Zipf(s=1.0) stream over 65 symbols stands in for the
  Shakespeare corpus (absent); batches are drawn as Dataset::sample_from
  (src/data.rs:174-191) with the xorshift generator seeded 42 + 1295
  (src/main.rs:420-424).

On the GPU arm every LayerNorm (ln_1, ln_2, ln_f), every dense layer
(c_attn, c_proj, out_proj, squeeze, process_1, lm_head), the attention and
the Kerr-ODE run through this library; the embedding lookup, residual adds,
PerBandLinear's 2x2 band maps, GELU, cross-entropy, clipping and Adam are
torch elementwise work.  lm_head is padded from 65 to 68 rows (a multiple
of 4, which the dense-layer kernels require); the padded rows stay zero.
"""
import math

import numpy as np

MASK64 = (1 << 64) - 1
N_BANDS, N_HEAD, N_LAYERS, MAESTRO_DIM, BLOCK_SIZE, RK4_STEPS = 64, 4, 4, 16, 256, 8
N_EMBD = 2 * N_BANDS
VOCAB = 65
LR = 3e-4
N_ITERS_SCHEDULE = 3000


class XorShift64:
    """src/rng.rs:5-45."""

    def __init__(self, seed: int):
        self.state = seed & MASK64

    def next_u64(self) -> int:
        s = self.state
        s ^= (s << 13) & MASK64
        s ^= s >> 7
        s ^= (s << 17) & MASK64
        self.state = s
        return s

    def next_f32(self) -> np.float32:
        return np.float32(self.next_u64() >> 40) / np.float32(1 << 24)

    def uniform(self, limit: np.float32) -> np.float32:
        return (self.next_f32() * np.float32(2.0) - np.float32(1.0)) * np.float32(limit)

    def next_usize(self, n: int) -> int:
        return self.next_u64() % n


def _uniform_matrix(rng: XorShift64, rows: int, cols: int, limit) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    for i in range(rows):
        for j in range(cols):
            out[i, j] = rng.uniform(limit)
    return out


def _linear(rng, out_dim, in_dim):
    """init_linear (src/init.rs:9-16): U(+-1/sqrt(in_dim)) row by row, zero bias."""
    limit = np.float32(1.0) / np.sqrt(np.float32(in_dim))
    return _uniform_matrix(rng, out_dim, in_dim, limit), np.zeros(out_dim, np.float32)


def init_model(seed: int = 42):
    """init_model_ext(vocab 65, seed, default_128, dual_maestro = false)."""
    rng = XorShift64(seed)
    C, nb = N_EMBD, N_BANDS
    blocks = []
    for i in range(N_LAYERS):
        p = {"ln1_w": np.ones(C, np.float32), "ln1_b": np.zeros(C, np.float32),
             "ln2_w": np.ones(C, np.float32), "ln2_b": np.zeros(C, np.float32)}
        p["wa"], p["ba"] = _linear(rng, 3 * C, C)
        p["wp"], p["bp"] = _linear(rng, C, C)
        if i == 0:
            limit = np.float32(1.0) / np.sqrt(np.float32(2.0))
            bw = np.empty((nb, 2, 2), np.float32)
            for b in range(nb):
                for r in range(2):
                    for c in range(2):
                        bw[b, r, c] = rng.uniform(limit)
            p["band_w"], p["band_b"] = bw, np.zeros((nb, 2), np.float32)
        else:
            p["gamma_raw"] = np.full(nb, np.log(np.expm1(np.float32(0.1))), np.float32)
            p["omega"] = ((np.arange(nb, dtype=np.float32) + 1) / np.float32(nb)).astype(np.float32)
            p["alpha_beta"] = np.array([0.1, 0.1], np.float32)
            p["wsq"], p["bsq"] = _linear(rng, MAESTRO_DIM, C)
            p["wpr"], p["bpr"] = _linear(rng, C, MAESTRO_DIM)
        p["wo"], p["bo"] = _linear(rng, C, C)
        blocks.append(p)
    limit = np.float32(1.0) / np.sqrt(np.float32(C))
    lm_head = _uniform_matrix(rng, VOCAB, C, limit)
    return blocks, {"lnf_w": np.ones(C, np.float32), "lnf_b": np.zeros(C, np.float32), "lm_head": lm_head}


def param_order(blocks):
    """Names of the trainable parameters in flatten_params order
    (src/optim.rs:185-240): per block ln_1, c_attn, c_proj, ln_2, FFN; then
    ln_f and lm_head."""
    order = []
    for i, p in enumerate(blocks):
        names = ["ln1_w", "ln1_b", "wa", "ba", "wp", "bp", "ln2_w", "ln2_b"]
        if "band_w" in p:
            names += ["band_w", "band_b", "wo", "bo"]
        else:
            names += ["gamma_raw", "omega", "alpha_beta", "wsq", "bsq", "wpr", "bpr", "wo", "bo"]
        order += [(i, n) for n in names]
    return order + [(None, "lnf_w"), (None, "lnf_b"), (None, "lm_head")]


def embeddings():
    """(wte [65][128], wpe [256][128]): build_harmonic_table_sized and
    build_positional_table (src/model.rs:104-135), in f32."""
    C, nh = N_EMBD, N_EMBD // 2
    scale = np.float32(1.0) / np.sqrt(np.float32(nh))
    pi = np.float32(math.pi)
    wte = np.zeros((VOCAB, C), np.float32)
    for c in range(VOCAB):
        theta = np.float32(c) * np.float32(2.0) * pi / np.float32(VOCAB)
        for h in range(nh):
            angle = np.float32(h + 1) * theta
            wte[c, 2 * h] = np.cos(angle) * scale
            wte[c, 2 * h + 1] = np.sin(angle) * scale
    wpe = np.zeros((BLOCK_SIZE, C), np.float32)
    for pos in range(BLOCK_SIZE):
        for h in range(nh):
            freq = np.float32(1.0) / np.power(np.float32(10000.0), np.float32(2.0 * h) / np.float32(C))
            wpe[pos, 2 * h] = np.cos(np.float32(pos) * freq) * scale
            wpe[pos, 2 * h + 1] = np.sin(np.float32(pos) * freq) * scale
    return wte, wpe


def token_stream(n: int = 1_000_000, s: float = 1.0, seed: int = 42) -> np.ndarray:
    """Seeded Zipf(s) ids over the 65 symbols (rank r has weight 1/(r+1)^s)."""
    w = 1.0 / np.arange(1, VOCAB + 1, dtype=np.float64) ** s
    return np.random.default_rng(seed).choice(VOCAB, size=n, p=w / w.sum()).astype(np.int64)


def sample_batch(data: np.ndarray, rng: XorShift64, B: int, T: int):
    """Dataset::sample_from (src/data.rs:174-191)."""
    max_start = len(data) - T - 1
    starts = [rng.next_usize(max_start) for _ in range(B)]
    x = np.stack([data[s:s + T] for s in starts])
    y = np.stack([data[s + 1:s + T + 1] for s in starts])
    return x, y


def active_bands(it: int, n_iters: int = N_ITERS_SCHEDULE) -> int:
    """CurriculumSchedule::default_3stage(64).active_bands (src/train.rs:29-69)."""
    cumulative = np.float32(0.0)
    for bands, frac in ((8, 0.333), (24, 0.333), (N_BANDS, 0.334)):
        cumulative = np.float32(cumulative + np.float32(frac))
        if it < int(np.float32(cumulative * np.float32(n_iters))):
            return bands
    return N_BANDS


SQRT_2_PI = np.float32(math.sqrt(2.0 / math.pi))


def gelu(x):
    """src/model.rs:75-77 (tanh approximation)."""
    x = np.asarray(x, np.float32)
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(SQRT_2_PI * (x + np.float32(0.044715) * x * x * x))))


def gelu_backward(dy, x):
    """src/backward.rs:132-147."""
    x = np.asarray(x, np.float32)
    t = np.tanh(SQRT_2_PI * (x + np.float32(0.044715) * x * x * x))
    sech2 = np.float32(1.0) - t * t
    d_inner = SQRT_2_PI * (np.float32(1.0) + np.float32(3.0 * 0.044715) * x * x)
    return (dy * (np.float32(0.5) * (np.float32(1.0) + t) + np.float32(0.5) * x * sech2 * d_inner)).astype(np.float32)


def cross_entropy(logits, targets):
    """Per-sequence mean cross-entropy and its gradient (src/pipeline.rs:369-386,
    src/backward.rs:159-170): d_logits = (softmax - onehot) / T."""
    B, T, V = logits.shape
    m = logits.max(-1, keepdims=True)
    e = np.exp(logits - m)
    s = e.sum(-1, keepdims=True)
    p = (e / s).astype(np.float32)
    loss = -np.log(np.take_along_axis(p, targets[..., None], -1)[..., 0]).mean(-1)  # [B]
    d = p.copy()
    np.put_along_axis(d, targets[..., None], np.take_along_axis(d, targets[..., None], -1) - 1, -1)
    return loss.astype(np.float32), (d / np.float32(T)).astype(np.float32)


class Adam:
    """src/optim.rs:9-83, one state per named parameter."""

    def __init__(self, lr=LR):
        self.lr, self.b1, self.b2, self.eps, self.t = np.float32(lr), np.float32(0.9), np.float32(0.999), \
            np.float32(1e-8), 0
        self.m, self.v = {}, {}

    def step(self, params: dict, grads: dict):
        self.t += 1
        bc1 = np.float32(1.0) - self.b1 ** np.float32(self.t)
        bc2 = np.float32(1.0) - self.b2 ** np.float32(self.t)
        for k, g in grads.items():
            m = self.m.get(k, np.zeros_like(g))
            v = self.v.get(k, np.zeros_like(g))
            m = (self.b1 * m + (np.float32(1.0) - self.b1) * g).astype(np.float32)
            v = (self.b2 * v + (np.float32(1.0) - self.b2) * g * g).astype(np.float32)
            self.m[k], self.v[k] = m, v
            params[k] = (params[k] - self.lr * (m / bc1) / (np.sqrt(v / bc2) + self.eps)).astype(np.float32)


def clip_scale(grads: dict, order) -> np.float32:
    """clip_grad_norm(grads, 1.0) (src/optim.rs:76-83): the factor applied to
    every gradient, from the f32 sequential sum of squares in flatten order."""
    flat = np.concatenate([grads[k].ravel() for k in order]).astype(np.float32)
    norm = np.sqrt(np.add.accumulate(flat * flat, dtype=np.float32)[-1])
    return np.float32(1.0) / norm if norm > np.float32(1.0) else np.float32(1.0)


def train_oracle(n_steps: int, B: int = 4, T: int = 64, seed: int = 42):
    """Losses of n_steps training steps on the oracle."""
    from oracle import oracle

    blocks, top = init_model(seed)
    wte, wpe = embeddings()
    data = token_stream()
    rng = XorShift64(seed + 1295)
    C, M, H = N_EMBD, B * T, N_HEAD
    params = {f"{i}.{k}": v for i, p in enumerate(blocks) for k, v in p.items()}
    params.update(top)
    order = [f"{i}.{n}" if i is not None else n for i, n in param_order(blocks)]
    adam = Adam()
    losses = []
    for it in range(n_steps):
        tok, tgt = sample_batch(data, rng, B, T)
        h = (wte[tok] + wpe[:T][None]).astype(np.float32)
        h[..., 2 * active_bands(it):] = 0.0
        h = h.reshape(M, C)
        caches = []
        for i in range(N_LAYERS):
            P = lambda k: params[f"{i}.{k}"]  # noqa: E731
            x1 = oracle.layernorm_forward(h, P("ln1_w"), P("ln1_b"))
            qkv = oracle.linear_forward(x1, P("wa"), P("ba")).reshape(B, T, 3 * C)
            q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
            o, att, _ = oracle.forward(q, k, v, H)
            o = o.reshape(M, C)
            h1 = h + oracle.linear_forward(o, P("wp"), P("bp"))
            x2 = oracle.layernorm_forward(h1, P("ln2_w"), P("ln2_b"))
            if i == 0:
                bw, bb = P("band_w"), P("band_b")
                r, s = x2[:, 0::2], x2[:, 1::2]
                bands = np.empty_like(x2)
                bands[:, 0::2] = bw[:, 0, 0] * r + bw[:, 1, 0] * s + bb[:, 0]
                bands[:, 1::2] = bw[:, 0, 1] * r + bw[:, 1, 1] * s + bb[:, 1]
                comb, extra = bands, None
            else:
                ab = P("alpha_beta")
                kerr = oracle.kerr_ode_forward(x2, P("gamma_raw"), P("omega"), ab[0], ab[1], RK4_STEPS)
                sq = oracle.linear_forward(x2, P("wsq"), P("bsq"))
                act = gelu(sq)
                comb = kerr + oracle.linear_forward(act, P("wpr"), P("bpr"))
                extra = (sq, act)
            ffn = oracle.linear_forward(comb, P("wo"), P("bo"))
            caches.append((h, x1, qkv, att, o, h1, x2, comb, extra))
            h = h1 + ffn
        nf = oracle.layernorm_forward(h, params["lnf_w"], params["lnf_b"])
        logits = oracle.linear_forward(nf, params["lm_head"], None).reshape(B, T, VOCAB)
        loss, dlog = cross_entropy(logits, tgt)
        losses.append(float(loss.mean()))
        dlog = (dlog / np.float32(B)).reshape(M, VOCAB)  # batch mean of the summed gradients
        g = {}
        d_nf = oracle.linear_backward_dx(dlog, params["lm_head"])
        g["lm_head"], _ = oracle.linear_backward_dw(dlog, nf)
        dh, g["lnf_w"], g["lnf_b"] = oracle.layernorm_backward(d_nf, h, params["lnf_w"])
        for i in reversed(range(N_LAYERS)):
            P = lambda k: params[f"{i}.{k}"]  # noqa: E731
            hin, x1, qkv, att, o, h1, x2, comb, extra = caches[i]
            d_comb = oracle.linear_backward_dx(dh, P("wo"))
            g[f"{i}.wo"], g[f"{i}.bo"] = oracle.linear_backward_dw(dh, comb)
            if i == 0:
                bw = P("band_w")
                r, s = x2[:, 0::2], x2[:, 1::2]
                dr, ds = d_comb[:, 0::2], d_comb[:, 1::2]
                gbw = np.empty_like(bw)
                gbw[:, 0, 0] = (dr * r).sum(0)
                gbw[:, 0, 1] = (ds * r).sum(0)
                gbw[:, 1, 0] = (dr * s).sum(0)
                gbw[:, 1, 1] = (ds * s).sum(0)
                g["0.band_w"] = gbw
                g["0.band_b"] = np.stack([dr.sum(0), ds.sum(0)], -1).astype(np.float32)
                dx2 = np.empty_like(x2)
                dx2[:, 0::2] = bw[:, 0, 0] * dr + bw[:, 0, 1] * ds
                dx2[:, 1::2] = bw[:, 1, 0] * dr + bw[:, 1, 1] * ds
            else:
                ab = P("alpha_beta")
                dx2, g[f"{i}.gamma_raw"], g[f"{i}.omega"], da, db = oracle.kerr_ode_backward(
                    d_comb, x2, P("gamma_raw"), P("omega"), ab[0], ab[1], RK4_STEPS)
                g[f"{i}.alpha_beta"] = np.array([da, db], np.float32)
                sq, act = extra
                d_act = oracle.linear_backward_dx(d_comb, P("wpr"))
                g[f"{i}.wpr"], g[f"{i}.bpr"] = oracle.linear_backward_dw(d_comb, act)
                d_sq = gelu_backward(d_act, sq)
                dx2 = dx2 + oracle.linear_backward_dx(d_sq, P("wsq"))
                g[f"{i}.wsq"], g[f"{i}.bsq"] = oracle.linear_backward_dw(d_sq, x2)
            dln2, g[f"{i}.ln2_w"], g[f"{i}.ln2_b"] = oracle.layernorm_backward(dx2, h1, P("ln2_w"))
            dh1 = dh + dln2
            d_o = oracle.linear_backward_dx(dh1, P("wp"))
            g[f"{i}.wp"], g[f"{i}.bp"] = oracle.linear_backward_dw(dh1, o)
            q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
            dq, dk, dv = oracle.backward(d_o.reshape(B, T, C), q, k, v, att, H)
            dqkv = np.concatenate([dq, dk, dv], axis=-1).reshape(M, 3 * C)
            dx1 = oracle.linear_backward_dx(dqkv, P("wa"))
            g[f"{i}.wa"], g[f"{i}.ba"] = oracle.linear_backward_dw(dqkv, x1)
            dln1, g[f"{i}.ln1_w"], g[f"{i}.ln1_b"] = oracle.layernorm_backward(dx1, hin, P("ln1_w"))
            dh = dh1 + dln1
        c = clip_scale(g, order)
        adam.step(params, {k: (v * c).astype(np.float32) for k, v in g.items()})
    return losses


def train_gpu(n_steps: int, B: int = 4, T: int = 64, seed: int = 42, device: int = 0):
    """Losses of n_steps training steps with every path operator on this
    library's kernels (the rest in torch on the same device)."""
    import torch

    import kerr_attn

    dev = torch.device("cuda", device)
    blocks, top = init_model(seed)
    wte, wpe = embeddings()
    data = token_stream()
    rng = XorShift64(seed + 1295)
    C, M, H, VP = N_EMBD, B * T, N_HEAD, 68
    params = {f"{i}.{k}": torch.from_numpy(v.copy()).to(dev) for i, p in enumerate(blocks) for k, v in p.items()}
    lm = np.zeros((VP, C), np.float32)
    lm[:VOCAB] = top["lm_head"]
    params["lm_head"] = torch.from_numpy(lm).to(dev)
    params["lnf_w"] = torch.from_numpy(top["lnf_w"].copy()).to(dev)
    params["lnf_b"] = torch.from_numpy(top["lnf_b"].copy()).to(dev)
    order = [f"{i}.{n}" if i is not None else n for i, n in param_order(blocks)]
    wte_d, wpe_d = torch.from_numpy(wte).to(dev), torch.from_numpy(wpe).to(dev)
    m_state = {k: torch.zeros_like(v) for k, v in params.items()}
    v_state = {k: torch.zeros_like(v) for k, v in params.items()}
    ctx = kerr_attn.Context(device)
    e = lambda *s: torch.empty(*s, device=dev)  # noqa: E731
    s2p = float(SQRT_2_PI)

    def gelu_t(x):
        return 0.5 * x * (1.0 + torch.tanh(s2p * (x + 0.044715 * x * x * x)))

    def gelu_bwd_t(dy, x):
        t = torch.tanh(s2p * (x + 0.044715 * x * x * x))
        return dy * (0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * (s2p * (1.0 + 3.0 * 0.044715 * x * x)))

    def lin(x, w, b, n_out):
        y = e(x.shape[0], n_out)
        kerr_attn.linear_fwd(ctx, x, w, b, y)
        return y

    def lin_dx(dy, w, n_in):
        dx = e(dy.shape[0], n_in)
        kerr_attn.linear_bwd_dx(ctx, dy, w, dx)
        return dx

    def lin_dw(dy, x, w, with_bias=True):
        dw = torch.empty_like(w)
        db = e(w.shape[0]) if with_bias else None
        kerr_attn.linear_bwd_dw(ctx, dy, x, dw, db, accumulate=False)
        return dw, db

    def ln(x, w, b):
        y = torch.empty_like(x)
        kerr_attn.layernorm_fwd(ctx, x, w, b, y)
        return y

    def ln_bwd(dy, x, w):
        dx, dw, db = torch.empty_like(x), torch.empty_like(w), torch.empty_like(w)
        kerr_attn.layernorm_bwd(ctx, dy, x, w, dx, dw, db, accumulate=False)
        return dx, dw, db

    losses = []
    try:
        for it in range(n_steps):
            tok, tgt = sample_batch(data, rng, B, T)
            tok_d = torch.from_numpy(tok).to(dev)
            h = wte_d[tok_d] + wpe_d[:T][None]
            h[..., 2 * active_bands(it):] = 0.0
            h = h.reshape(M, C).contiguous()
            caches = []
            for i in range(N_LAYERS):
                P = lambda k: params[f"{i}.{k}"]  # noqa: E731
                x1 = ln(h, P("ln1_w"), P("ln1_b"))
                qkv = lin(x1, P("wa"), P("ba"), 3 * C).view(B, T, 3 * C)
                q, k, v = kerr_attn.split_qkv(qkv, C)
                o, lse = e(B, T, C), e(B, H, T)
                kerr_attn.fwd(ctx, q, k, v, o, lse, H)
                h1 = h + lin(o.view(M, C), P("wp"), P("bp"), C)
                x2 = ln(h1, P("ln2_w"), P("ln2_b"))
                if i == 0:
                    bw, bb = P("band_w"), P("band_b")
                    r, s = x2[:, 0::2], x2[:, 1::2]
                    comb = torch.empty_like(x2)
                    comb[:, 0::2] = bw[:, 0, 0] * r + bw[:, 1, 0] * s + bb[:, 0]
                    comb[:, 1::2] = bw[:, 0, 1] * r + bw[:, 1, 1] * s + bb[:, 1]
                    extra = None
                else:
                    kerr = e(M, C)
                    kerr_attn.kerr_ode_fwd(ctx, x2, P("gamma_raw"), P("omega"), P("alpha_beta"), kerr, RK4_STEPS)
                    sq = lin(x2, P("wsq"), P("bsq"), MAESTRO_DIM)
                    act = gelu_t(sq)
                    comb = kerr + lin(act, P("wpr"), P("bpr"), C)
                    extra = (sq, act)
                h_next = h1 + lin(comb, P("wo"), P("bo"), C)
                caches.append((h, x1, qkv, o, lse, h1, x2, comb, extra))
                h = h_next
            nf = ln(h, params["lnf_w"], params["lnf_b"])
            logits = lin(nf, params["lm_head"], None, VP)[:, :VOCAB].reshape(B, T, VOCAB)
            tgt_d = torch.from_numpy(tgt).to(dev)
            p = torch.softmax(logits, -1)
            loss = -torch.log(p.gather(-1, tgt_d[..., None])[..., 0]).mean(-1)
            losses.append(float(loss.mean().item()))
            dlog = p.clone()
            dlog.scatter_add_(-1, tgt_d[..., None], -torch.ones_like(tgt_d[..., None], dtype=p.dtype))
            dlog = (dlog / (T * B)).reshape(M, VOCAB)
            dlp = torch.zeros(M, VP, device=dev)
            dlp[:, :VOCAB] = dlog
            g = {}
            d_nf = lin_dx(dlp, params["lm_head"], C)
            g["lm_head"], _ = lin_dw(dlp, nf, params["lm_head"], with_bias=False)
            dh, g["lnf_w"], g["lnf_b"] = ln_bwd(d_nf, h, params["lnf_w"])
            for i in reversed(range(N_LAYERS)):
                P = lambda k: params[f"{i}.{k}"]  # noqa: E731
                hin, x1, qkv, o, lse, h1, x2, comb, extra = caches[i]
                d_comb = lin_dx(dh, P("wo"), C)
                g[f"{i}.wo"], g[f"{i}.bo"] = lin_dw(dh, comb, P("wo"))
                if i == 0:
                    bw = P("band_w")
                    r, s = x2[:, 0::2], x2[:, 1::2]
                    dr, ds = d_comb[:, 0::2], d_comb[:, 1::2]
                    gbw = torch.empty_like(bw)
                    gbw[:, 0, 0] = (dr * r).sum(0)
                    gbw[:, 0, 1] = (ds * r).sum(0)
                    gbw[:, 1, 0] = (dr * s).sum(0)
                    gbw[:, 1, 1] = (ds * s).sum(0)
                    g["0.band_w"] = gbw
                    g["0.band_b"] = torch.stack([dr.sum(0), ds.sum(0)], -1)
                    dx2 = torch.empty_like(x2)
                    dx2[:, 0::2] = bw[:, 0, 0] * dr + bw[:, 0, 1] * ds
                    dx2[:, 1::2] = bw[:, 1, 0] * dr + bw[:, 1, 1] * ds
                else:
                    dx2 = e(M, C)
                    g[f"{i}.gamma_raw"], g[f"{i}.omega"], g[f"{i}.alpha_beta"] = e(N_BANDS), e(N_BANDS), e(2)
                    kerr_attn.kerr_ode_bwd(ctx, d_comb, x2, P("gamma_raw"), P("omega"), P("alpha_beta"), dx2,
                                           g[f"{i}.gamma_raw"], g[f"{i}.omega"], g[f"{i}.alpha_beta"], RK4_STEPS,
                                           accumulate=False)
                    sq, act = extra
                    d_act = lin_dx(d_comb, P("wpr"), MAESTRO_DIM)
                    g[f"{i}.wpr"], g[f"{i}.bpr"] = lin_dw(d_comb, act, P("wpr"))
                    d_sq = gelu_bwd_t(d_act, sq)
                    dx2 = dx2 + lin_dx(d_sq, P("wsq"), C)
                    g[f"{i}.wsq"], g[f"{i}.bsq"] = lin_dw(d_sq, x2, P("wsq"))
                dln2, g[f"{i}.ln2_w"], g[f"{i}.ln2_b"] = ln_bwd(dx2, h1, P("ln2_w"))
                dh1 = dh + dln2
                d_o = lin_dx(dh1, P("wp"), C).view(B, T, C)
                g[f"{i}.wp"], g[f"{i}.bp"] = lin_dw(dh1, o.view(M, C), P("wp"))
                q, k, v = kerr_attn.split_qkv(qkv, C)
                dqkv = e(B, T, 3 * C)
                dq, dk, dv = kerr_attn.split_qkv(dqkv, C)
                kerr_attn.bwd(ctx, q, k, v, o, d_o, lse, dq, dk, dv, H)
                dx1 = lin_dx(dqkv.view(M, 3 * C), P("wa"), C)
                g[f"{i}.wa"], g[f"{i}.ba"] = lin_dw(dqkv.view(M, 3 * C), x1, P("wa"))
                dln1, g[f"{i}.ln1_w"], g[f"{i}.ln1_b"] = ln_bwd(dx1, hin, P("ln1_w"))
                dh = dh1 + dln1
            norm = torch.sqrt(sum((g[k].double() ** 2).sum() for k in order)).float()
            c = (1.0 / norm) if norm > 1.0 else torch.tensor(1.0, device=dev)
            t = it + 1
            bc1, bc2 = 1.0 - 0.9 ** t, 1.0 - 0.999 ** t
            for k in order:
                gk = g[k] * c
                m_state[k].mul_(0.9).add_(gk, alpha=0.1)
                v_state[k].mul_(0.999).addcmul_(gk, gk, value=0.001)
                params[k] -= LR * (m_state[k] / bc1) / (torch.sqrt(v_state[k] / bc2) + 1e-8)
        torch.cuda.synchronize(dev)
        ctx.check_device()
    finally:
        ctx.close()
    return losses
