"""Independent float64 Kerr-ODE for the tests: the same ODE (src/model.rs:
778-843) written with torch tensor ops, differentiated by autograd.  This is
how the reference validates its own Kerr-ODE backward (src/grad_test.rs:
50-174 compares it against PyTorch autograd); its recorded vectors
(reference/gradient_test.bin) are not in the reference tree, so the
comparison is rerun here."""
import numpy as np
import torch


def kerr_ode(x, gamma_raw, omega, alpha, beta, n_steps):
    """x [M, 2 nb] (interleaved r, s) -> y [M, 2 nb]; any float dtype, autograd-able."""
    r, s = x[:, 0::2], x[:, 1::2]
    gamma = torch.where(gamma_raw > 20, gamma_raw, torch.log1p(torch.exp(torch.clamp(gamma_raw, max=20))))
    dt = 1.0 / n_steps

    def f(r, s):
        m = r * r + s * s
        z = torch.zeros_like(m[:, :2])
        mp = torch.cat([z, m, z], dim=1)
        ns = mp[:, 0:-4] + mp[:, 1:-3] + mp[:, 3:-1] + mp[:, 4:]
        phi = omega + alpha * m + beta * ns
        return -gamma * r - phi * s, -gamma * s + phi * r

    for _ in range(n_steps):
        a1, b1 = f(r, s)
        a2, b2 = f(r + 0.5 * dt * a1, s + 0.5 * dt * b1)
        a3, b3 = f(r + 0.5 * dt * a2, s + 0.5 * dt * b2)
        a4, b4 = f(r + dt * a3, s + dt * b3)
        r = r + dt / 6 * (a1 + 2 * a2 + 2 * a3 + a4)
        s = s + dt / 6 * (b1 + 2 * b2 + 2 * b3 + b4)
    return torch.stack([r, s], dim=2).reshape(x.shape)


def forward_backward(x, dy, gamma_raw, omega, alpha, beta, n_steps):
    """float64 (y, dx, d_gamma_raw, d_omega, d_alpha, d_beta) as numpy / floats."""
    X = torch.tensor(np.asarray(x, np.float64), requires_grad=True)
    G = torch.tensor(np.asarray(gamma_raw, np.float64), requires_grad=True)
    O = torch.tensor(np.asarray(omega, np.float64), requires_grad=True)
    A = torch.tensor(float(alpha), dtype=torch.float64, requires_grad=True)
    B = torch.tensor(float(beta), dtype=torch.float64, requires_grad=True)
    Y = kerr_ode(X, G, O, A, B, n_steps)
    Y.backward(torch.tensor(np.asarray(dy, np.float64)))
    return (Y.detach().numpy(), X.grad.numpy(), G.grad.numpy(), O.grad.numpy(), A.grad.item(), B.grad.item())


def reference_cases():
    """The Kerr-ODE inputs of the reference's own GPU-vs-CPU checks
    (src/gpu_validate.rs:81-105, :107-157, :159-208), each as
    (name, x [M, 2 nb], gamma_raw, omega, alpha, beta, n_steps).  The reference
    accepts a maximum absolute difference below 1e-4 on them."""
    cases = []
    nb = 64
    k = np.arange(nb, dtype=np.float32)
    x = np.empty((1, 2 * nb), np.float32)
    x[0, 0::2] = np.cos(k * np.float32(0.1)) * np.float32(0.5)
    x[0, 1::2] = np.sin(k * np.float32(0.1)) * np.float32(0.5)
    cases.append(("kerr_ode_64_bands_1_pos", x, np.float32(-2.0) + k * np.float32(0.05), k / np.float32(nb),
                  0.1, 0.1, 8))
    for nb, n_pos, step, g_slope, n_steps in ((384, 4, 0.003, 0.01, 16), (64, 4, 0.01, 0.05, 8)):
        k = np.arange(nb, dtype=np.float32)
        i = np.arange(n_pos * 2 * nb, dtype=np.float32).reshape(n_pos, 2 * nb)
        x = np.sin(i * np.float32(step)).astype(np.float32)
        cases.append((f"fused_rk4_{nb}_bands_{n_pos}_pos", x, np.float32(-2.0) + k * np.float32(g_slope),
                      k / np.float32(nb), 0.1, 0.1, n_steps))
    return cases


def init_params(nb, seed=None):
    """The reference's initial KerrWeights (src/init.rs:50-61): gamma_raw =
    softplus^-1(0.1), omega_k = (k+1)/nb, alpha = beta = 0.1; with a seed,
    perturbed as training would move them."""
    gamma_raw = np.full(nb, np.log(np.expm1(0.1)), np.float32)
    omega = ((np.arange(nb) + 1) / nb).astype(np.float32)
    alpha, beta = 0.1, 0.1
    if seed is not None:
        rng = np.random.default_rng(seed)
        gamma_raw = (gamma_raw + 0.5 * rng.standard_normal(nb)).astype(np.float32)
        omega = (omega + 0.1 * rng.standard_normal(nb)).astype(np.float32)
        alpha, beta = 0.1 + 0.02 * float(rng.standard_normal()), 0.1 + 0.02 * float(rng.standard_normal())
    return gamma_raw, omega, float(np.float32(alpha)), float(np.float32(beta))
