"""CPU oracle of the OSCAR INT2 path. TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs;
the product package ``oscar_new_b200`` must never import it.
"""
