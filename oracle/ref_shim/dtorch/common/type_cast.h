// Shim (oracle build): checked downcast used by ThreadGroup::SetStream.
#pragma once
namespace dtorch {
template <typename Derived, typename Base>
inline Derived* DerivedCast(Base* p) { return dynamic_cast<Derived*>(p); }
}  // namespace dtorch
