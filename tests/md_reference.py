"""Reference integrators for the MD driver tests (test infrastructure).

A plain numpy restatement of LAMMPS' `fix nve`, `fix nvt` and `fix npt iso` step
order in metal units, with the Nose-Hoover chains of FixNH
(nhc_temp_integrate / nhc_press_integrate, one Suzuki-Yoshida stage, no drag)
and the MTK barostat terms (nh_omega_dot, nh_v_press, remap about the origin).
The force callback is the CPU oracle, so the GPU driver's trajectory can be
compared step for step.
"""
import numpy as np

MVV2E = 1.0364269e-4
FTM2V = 1.0 / MVV2E
BOLTZ = 8.617343e-5


def temperature(v, m):
    dof = 3 * len(m) - 3
    return float((m[:, None] * v * v).sum() * MVV2E / (dof * BOLTZ))


class Chain:
    def __init__(self, dof, t_target, t_damp, M, dt):
        w = 1.0 / t_damp
        self.M = M
        self.dof_boltz = dof * BOLTZ
        self.ke_target = dof * BOLTZ * t_target
        self.boltz_t = BOLTZ * t_target
        self.mass = np.array([self.ke_target / w ** 2] + [self.boltz_t / w ** 2] * (M - 1))
        self.eta = np.zeros(M)
        self.eta_dot = np.zeros(M + 1)
        self.eta_dotdot = np.zeros(M)
        for i in range(1, M):
            self.eta_dotdot[i] = (self.mass[i - 1] * self.eta_dot[i - 1] ** 2 - self.boltz_t) / self.mass[i]
        self.dt4, self.dt8, self.dthalf = 0.25 * dt, 0.125 * dt, 0.5 * dt

    def half(self, t_current):
        """One chain half-step; returns (velocity factor, rescaled temperature)."""
        M, ed, edd = self.M, self.eta_dot, self.eta_dotdot
        edd[0] = (self.dof_boltz * t_current - self.ke_target) / self.mass[0]
        for i in range(M - 1, 0, -1):
            x = np.exp(-self.dt8 * ed[i + 1])
            ed[i] = (ed[i] * x + edd[i] * self.dt4) * x
        x = np.exp(-self.dt8 * ed[1])
        ed[0] = (ed[0] * x + edd[0] * self.dt4) * x
        factor = np.exp(-self.dthalf * ed[0])
        t_current *= factor * factor
        edd[0] = (self.dof_boltz * t_current - self.ke_target) / self.mass[0]
        self.eta += self.dthalf * ed[:M]
        ed[0] = (ed[0] * x + edd[0] * self.dt4) * x
        for i in range(1, M):
            x = np.exp(-self.dt8 * ed[i + 1])
            edd[i] = (self.mass[i - 1] * ed[i - 1] ** 2 - self.boltz_t) / self.mass[i]
            ed[i] = (ed[i] * x + edd[i] * self.dt4) * x
        return factor, t_current

    def energy(self):
        e = self.ke_target * self.eta[0] + self.boltz_t * self.eta[1:self.M].sum()
        return float(e + 0.5 * (self.mass * self.eta_dot[:self.M] ** 2).sum())


def run(x, v, m, force, dt, nsteps, chain=None):
    """Velocity Verlet (+ chain); force(x) -> (energy, forces)."""
    x, v = x.copy(), v.copy()
    e, f = force(x)
    t_current = temperature(v, m)
    dtf = 0.5 * dt * FTM2V
    for _ in range(nsteps):
        if chain is not None:
            s, t_current = chain.half(t_current)
            v *= s
        v += dtf * f / m[:, None]
        x += dt * v
        e, f = force(x)
        v += dtf * f / m[:, None]
        t_current = temperature(v, m)
        if chain is not None:
            s, t_current = chain.half(t_current)
            v *= s
    return x, v, e


NKTV2P = 1.6021765e6


class BaroChain(Chain):
    """Barostat chain: masses kB T0 / wp^2, kinetic energy 3 W omega_dot^2 against kB T0."""

    def __init__(self, t_target, p_damp, M, dt):
        wp = 1.0 / p_damp
        kt = BOLTZ * t_target
        self.M = M
        self.kt = kt
        self.mass = np.full(M, kt / wp ** 2)
        self.eta = np.zeros(M)
        self.eta_dot = np.zeros(M + 1)
        self.eta_dotdot = np.zeros(M)
        for i in range(1, M):
            self.eta_dotdot[i] = (self.mass[i - 1] * self.eta_dot[i - 1] ** 2 - kt) / self.mass[i]
        self.dt4, self.dt8, self.dthalf = 0.25 * dt, 0.125 * dt, 0.5 * dt

    def press(self, omega_dot, w_mass):
        M, ed, edd = self.M, self.eta_dot, self.eta_dotdot
        edd[0] = (3 * w_mass * omega_dot ** 2 - self.kt) / self.mass[0]
        for i in range(M - 1, 0, -1):
            x = np.exp(-self.dt8 * ed[i + 1])
            ed[i] = (ed[i] * x + edd[i] * self.dt4) * x
        x = np.exp(-self.dt8 * ed[1])
        ed[0] = (ed[0] * x + edd[0] * self.dt4) * x
        self.eta += self.dthalf * ed[:M]
        omega_dot *= np.exp(-self.dthalf * ed[0])
        edd[0] = (3 * w_mass * omega_dot ** 2 - self.kt) / self.mass[0]
        ed[0] = (ed[0] * x + edd[0] * self.dt4) * x
        for i in range(1, M):
            x = np.exp(-self.dt8 * ed[i + 1])
            edd[i] = (self.mass[i - 1] * ed[i - 1] ** 2 - self.kt) / self.mass[i]
            ed[i] = (ed[i] * x + edd[i] * self.dt4) * x
        return omega_dot


def run_npt(x, v, m, force, box, dt, nsteps, t_target, t_damp, tchain, p_target, p_damp, pchain):
    """fix npt iso (MTK); force(x, box) -> (energy, forces, virial 3x3).  Returns x, v, box, energy."""
    x, v, box = x.copy(), v.copy(), box.copy()
    n = len(m)
    dof = 3 * n - 3
    chain = Chain(dof, t_target, t_damp, tchain, dt)
    baro = BaroChain(t_target, p_damp, pchain, dt)
    kt = BOLTZ * t_target
    w_mass = (n + 1) * kt / (1.0 / p_damp) ** 2
    e, f, w = force(x, box)
    t_current = temperature(v, m)
    omega_dot = 0.0
    dtf, dthalf = 0.5 * dt * FTM2V, 0.5 * dt

    def omega_force(t_cur, vir_tr, omega_dot):
        vol = np.prod(np.diag(box))
        p_cur = (dof * BOLTZ * t_cur + vir_tr) / (3 * vol) * NKTV2P
        mtk1 = dof * BOLTZ * t_cur / (3 * n)
        return omega_dot + ((p_cur - p_target) * vol / (w_mass * NKTV2P) + mtk1 / w_mass) * dthalf

    for _ in range(nsteps):
        omega_dot = baro.press(omega_dot, w_mass)
        s, t_current = chain.half(t_current)
        v *= s
        omega_dot = omega_force(t_current, np.trace(w), omega_dot)
        fp = np.exp(-0.25 * dt * (omega_dot + omega_dot / n))
        v *= fp * fp
        v += dtf * f / m[:, None]
        ex = np.exp(dthalf * omega_dot)
        x = ex * (ex * x + dt * v)
        box = box * ex * ex
        e, f, w = force(x, box)
        v += dtf * f / m[:, None]
        v *= fp * fp
        t_current = temperature(v, m)
        omega_dot = omega_force(t_current, np.trace(w), omega_dot)
        s, t_current = chain.half(t_current)
        v *= s
        omega_dot = baro.press(omega_dot, w_mass)
    return x, v, box, e
