"""Model families written by ``pluggy_b200.synth.write_model``.

Each ``<name>.py`` here passed its own ``__main__`` scaffold and the model contract
check before its key was added to ``registry.json``; none was reviewed by a person.
"""
