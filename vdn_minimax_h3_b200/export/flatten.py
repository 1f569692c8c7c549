"""Flatten a module and its in-package import closure into ONE importable source file.

Reference parity: src/diffusers_export/export.py:51-111,244-295 (the published component
is a single modeling file: the package closure merged, import statements rewritten, the
definition order validated). This implementation works on the AST:

* the closure is every `vdn_minimax_h3_b200.*` module reached by top-level imports from
  the entry;
* modules are emitted in dependency order (a module after everything it imports);
* in-package imports are removed (their names are globals of the merged file); an import
  alias becomes an assignment at the top of the importing module's section; an in-package
  import inside a function body whose module is outside the closure becomes a `raise
  ImportError(...)` (that code path is not part of the component);
* `from __future__` lines are hoisted; stdlib / third-party imports stay in place;
* two modules defining the same top-level name with different source is a hard error
  (so a new collision fails the export instead of silently shadowing), identical
  definitions are kept once;
* anything the rewriter cannot map (a module-object import of the package, a relative
  import) is a hard error.
"""
import ast
import importlib.util
import os

PACKAGE = "vdn_minimax_h3_b200"


class FlattenError(RuntimeError):
    pass


def _module_file(name):
    spec = importlib.util.find_spec(name)
    if spec is None or not spec.origin or not spec.origin.endswith(".py"):
        raise FlattenError(f"cannot locate the source of {name}")
    return spec.origin


def _in_package(name):
    return name == PACKAGE or name.startswith(PACKAGE + ".")


def _check_import(node, where):
    if isinstance(node, ast.ImportFrom):
        if node.level:
            raise FlattenError(f"{where}: relative import is not supported")
        return node.module if node.module and _in_package(node.module) else None
    if isinstance(node, ast.Import):
        for a in node.names:
            if _in_package(a.name):
                raise FlattenError(f"{where}: `import {a.name}` (module object) cannot be "
                                   "flattened; import names from it")
    return None


def _top_level_deps(tree, where):
    deps = []
    for node in tree.body:
        mod = _check_import(node, where)
        if mod is not None:
            _assert_names_import(node, mod, where)
            deps.append(mod)
    return deps


def _assert_names_import(node, mod, where):
    for a in node.names:
        sub = f"{mod}.{a.name}"
        spec = importlib.util.find_spec(sub) if _is_package(mod) else None
        if spec is not None:
            raise FlattenError(f"{where}: `from {mod} import {a.name}` imports a module "
                               "object; import names from it")


def _is_package(mod):
    spec = importlib.util.find_spec(mod)
    return spec is not None and spec.submodule_search_locations is not None


def closure(entry):
    """Modules reached from `entry` by top-level in-package imports, dependencies first."""
    order, state = [], {}

    def visit(name, chain):
        if state.get(name) == "done":
            return
        if state.get(name) == "active":
            raise FlattenError("import cycle: " + " -> ".join(chain + [name]))
        state[name] = "active"
        path = _module_file(name)
        with open(path) as f:
            tree = ast.parse(f.read(), path)
        for dep in _top_level_deps(tree, name):
            visit(dep, chain + [name])
        state[name] = "done"
        order.append(name)

    visit(entry, [])
    return order


class _Rewriter(ast.NodeTransformer):
    """Drops in-package imports; nested imports of modules outside the closure raise."""

    def __init__(self, modules, where):
        self.modules = set(modules)
        self.where = where
        self.depth = 0
        self.aliases = []

    def _scope(self, node):
        self.depth += 1
        self.generic_visit(node)
        self.depth -= 1
        return node

    visit_FunctionDef = visit_AsyncFunctionDef = visit_ClassDef = _scope

    def visit_ImportFrom(self, node):
        mod = _check_import(node, self.where)
        if mod is None:
            return node
        if mod in self.modules:
            for a in node.names:
                if a.asname and a.asname != a.name:
                    self.aliases.append((a.asname, a.name, self.depth))
            if self.depth:
                # names are module globals of the merged file; keep local aliases working
                return [ast.Assign(targets=[ast.Name(a.asname, ast.Store())],
                                   value=ast.Name(a.name, ast.Load()))
                        for a in node.names if a.asname and a.asname != a.name] or ast.Pass()
            return None
        if self.depth == 0:
            raise FlattenError(f"{self.where}: top-level import of {mod}, outside the closure")
        msg = f"{mod} is not part of the exported component"
        return ast.Raise(exc=ast.Call(func=ast.Name("ImportError", ast.Load()),
                                      args=[ast.Constant(msg)], keywords=[]), cause=None)

    def visit_Import(self, node):
        _check_import(node, self.where)
        return node


def _defined_names(stmt):
    if isinstance(stmt, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
        return [stmt.name]
    names = []
    if isinstance(stmt, (ast.Assign, ast.AnnAssign)):
        targets = stmt.targets if isinstance(stmt, ast.Assign) else [stmt.target]
        for t in targets:
            for n in ast.walk(t):
                if isinstance(n, ast.Name):
                    names.append(n.id)
    return names


def flatten(entry, header=""):
    """-> merged source text of `entry` and its closure."""
    modules = closure(entry)
    future, sections, seen = set(), [], {}
    for name in modules:
        path = _module_file(name)
        with open(path) as f:
            src = f.read()
        tree = ast.parse(src, path)
        rw = _Rewriter(modules, name)
        body = []
        for stmt in tree.body:
            if isinstance(stmt, ast.ImportFrom) and stmt.module == "__future__":
                future.update(a.name for a in stmt.names)
                continue
            if (isinstance(stmt, ast.Expr) and isinstance(stmt.value, ast.Constant)
                    and isinstance(stmt.value.value, str) and not body):
                continue   # module docstring
            new = rw.visit(stmt)
            if new is None:
                continue
            stmts = new if isinstance(new, list) else [new]
            for s in stmts:
                dup = False
                for n in _defined_names(s):
                    text = ast.unparse(s)
                    if n in seen and seen[n][1] != text and n != "__all__":
                        raise FlattenError(f"top-level name {n!r} is defined by both "
                                           f"{seen[n][0]} and {name}")
                    if n in seen and seen[n][1] == text:
                        dup = True
                    seen.setdefault(n, (name, text))
                if not dup:
                    body.append(s)
        aliases = [ast.Assign(targets=[ast.Name(a, ast.Store())], value=ast.Name(n, ast.Load()))
                   for a, n, depth in rw.aliases if depth == 0]
        module = ast.Module(body=aliases + body, type_ignores=[])
        ast.fix_missing_locations(module)
        sections.append(f"# {'-' * 70}\n# from {name}\n" + ast.unparse(module))
    head = "".join(f"from __future__ import {n}\n" for n in sorted(future))
    out = head + (header.rstrip() + "\n\n" if header else "") + "\n\n\n".join(sections) + "\n"
    compile(out, "<flattened>", "exec")
    return out, modules


def write_flattened(entry, path, header=""):
    src, modules = flatten(entry, header)
    tmp = path + ".tmp"
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(tmp, "w") as f:
        f.write(src)
    os.replace(tmp, path)
    return modules
