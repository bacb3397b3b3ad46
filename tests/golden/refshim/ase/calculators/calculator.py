"""Stand-in of ``ase.calculators.calculator`` (test infrastructure only)."""

all_changes = ["positions", "numbers", "cell", "pbc", "initial_charges", "initial_magmoms"]


class Calculator:
    implemented_properties: list = []

    def __init__(self, *args, **kwargs):
        self.results = {}
        self.atoms = None
