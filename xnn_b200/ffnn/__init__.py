"""Force-field physics: polarizable multipole electrostatics with particle-mesh Ewald."""
