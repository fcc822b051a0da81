/* Host-side helper for the seeded synthetic trajectory generator (benchmark
 * configuration 4).  Integrates the 2-D overdamped Langevin equation in the
 * double-well potential U(x,y) = (x^2-1)^2 + y^2 with Euler-Maruyama:
 *     x <- x - dU/dx dt + sqrt(2 kT dt) xi_x,   y <- y - dU/dy dt + sqrt(2 kT dt) xi_y
 * using caller-supplied standard-normal increments xi (nsteps x 2, row-major),
 * and stores every keep-th state into out (nsteps/keep x 2).  Sequential by
 * nature, so it lives in C rather than in a Python loop. */
#include <math.h>

int fd_synth_langevin(const double* noise, long nsteps, double x, double y,
                      double dt, double kT, long keep, double* out) {
    if (!noise || !out || nsteps < 0 || keep <= 0) return 1;
    const double amp = sqrt(2.0 * kT * dt);
    long k = 0;
    for (long s = 0; s < nsteps; ++s) {
        const double gx = 4.0 * x * (x * x - 1.0);
        const double gy = 2.0 * y;
        x = x - gx * dt + amp * noise[2 * s];
        y = y - gy * dt + amp * noise[2 * s + 1];
        if ((s + 1) % keep == 0) {
            out[2 * k] = x;
            out[2 * k + 1] = y;
            ++k;
        }
    }
    return 0;
}
