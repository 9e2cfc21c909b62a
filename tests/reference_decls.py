"""Stand-ins for torchcst's chart and kernel declarations (attribute structure
only), for tests that run the plugin's Algorithm bodies where the reference
package is absent (the GPU box). ``tests/test_plugin_cpu.py`` checks that each
stand-in converts to the same native plan as the reference's own declaration
of the same layer, so the stand-ins cannot drift from the reference's shape.
"""

from types import SimpleNamespace as NS

import numpy as np


def f32(v):
    """torchcst declarations hold their scalars as float32 buffers read back."""
    return float(np.float32(v))


def chart(n, spacing=1.0, origin=0.0):
    return NS(kind="regular_grid", shape=(n,), spacing=(float(spacing),), origin=(float(origin),),
              geometry=NS(id="flat_torus"))


def profile(modes=8, base=1, merge=2):
    return NS(profile=NS(id="chebyshev", modes=modes), base_tile_sites=base, merge_factor=merge)


def rational_kernel(radius_max, *, radius_min=0.5, radius_birth=4.0, amplitude_max=32.0,
                    base=(1, 1), merge=(2, 2)):
    par = NS(id="rational_radius", radius_min=f32(radius_min), radius_birth=f32(radius_birth),
             radius_max=f32(radius_max), amplitude_max=f32(amplitude_max))
    return NS(profiles=(profile(8, base[0], merge[0]), profile(8, base[1], merge[1])),
              parameterization=par, revision=8, composition="separable",
              update=NS(settings=()), initialization=NS(settings=()))


def polar_kernel(*, amplitude_max=1.0, w_c=0.3, bounds=(0.5, 4.0, 50.0, 1.0), base_in=49,
                 kappa=3.0, upper_decay_power=1.0, radial_regularization=0.1):
    b = NS(minimum=f32(bounds[0]), birth=f32(bounds[1]), maximum=f32(bounds[2]),
           upper_floor=f32(bounds[3]))
    par = NS(id="polar_activity_radius", radius_envelope="rational",
             amplitude_max=f32(amplitude_max), w_c=f32(w_c), input_bounds=b, output_bounds=b,
             kappa=f32(kappa), lower_kappa=f32(kappa), upper_decay_power=f32(upper_decay_power))
    update = NS(settings=(("radial_regularization", f32(radial_regularization)),
                          ("activity_gain", 1.0), ("activity_mode", "finite_chord"),
                          ("dormant_expansion_rate", 0.0)))
    return NS(profiles=(profile(8, 1, 2), profile(8, base_in, 2)), parameterization=par,
              revision=7, composition="separable", update=update,
              initialization=NS(settings=(("alpha_init", 0.0),)))


def recipe(validate="sync"):
    return NS(validate=validate)
