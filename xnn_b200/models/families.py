"""Imports every model family so that their ``@register_model`` decorators run."""
from . import aimnet2, allegro, ani, bamboo, cace, cgcnn, cnn3d, d3, d4, dimenet, equiformer, equiformer_v2, et, gemnet, hdnnp, mace, megnet, nequip, painn, physnet, qet, qrnn, s2cnn, schnet, se3cnn, sgdml, spookynet, tensornet  # noqa: F401
from ..ffnn import amber, amoeba, byteff, byteff_pol, charmm, dreiding, opls, reaxff  # noqa: F401,E402  (classical and reactive force fields)
from ..sqm import nddo  # noqa: F401,E402  (semi-empirical quantum chemistry)
