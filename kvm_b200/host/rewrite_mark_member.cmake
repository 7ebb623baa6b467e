# cmake -DIN=<preprocessed> -DOUT=<rewritten> -P rewrite_mark_member.cmake
#
# Rewrites `struct ::kvm::ir::MarkMember` (a global qualifier before a
# class-key, which GCC rejects; produced by KVM_MARK_MEMBER in the reference's
# src/ir/any_of.h:76) to `struct kvm::ir::MarkMember` in a preprocessed
# translation unit. Nothing else changes.
file(READ "${IN}" text)
string(REPLACE "struct ::kvm::ir::MarkMember" "struct kvm::ir::MarkMember" text "${text}")
file(WRITE "${OUT}" "${text}")
file(REMOVE "${IN}")
