"""Reference integrators for the MD driver tests (test infrastructure).

A plain numpy restatement of LAMMPS' `fix nve` and `fix nvt` step order in metal
units, with the Nose-Hoover chain of FixNH::nhc_temp_integrate (one
Suzuki-Yoshida stage, no drag).  The force callback is the CPU oracle, so the
GPU driver's trajectory can be compared step for step.
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
