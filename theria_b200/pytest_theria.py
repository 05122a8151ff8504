"""pytest plugin: run a test suite written against ``theria`` on this library.

``pytest -p theria_b200.pytest_theria <theria checkout>/tests`` makes every
``import theria...`` in the collected files resolve to theria_b200 (see
``theria_b200.compat``), so the reference's own tests run unchanged.
"""

from theria_b200.compat import install_as_theria

install_as_theria()
