! Drop-in replacement of module matmul_cuda_fortran (matmul_cuda_fortran.cuf) over
! libq35.so: the same two procedures and arguments, callable from plain Fortran (no CUDA
! Fortran compiler needed).  The matrices stay resident on the GPU between calls with the
! same arrays (libq35's per-call cache).  The reference's fused kernel folds the scale
! into an fp32 accumulation; here the sum is exact int32, then Out = real(C) * scale
! (matmul_int4_groq.f90:58-69).  Optional stat= as in the other drop-ins.
! Compile after q35_status.f90.
module matmul_cuda_fortran
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float
    use iso_fortran_env, only: int8, int32, real32
    use q35_status, only: q35_check
    implicit none
    private
    public :: matmul_int4_cuda, matmul_int4_cuda_fused

    interface
        integer(c_int) function q35_matmul_int4_awq(A, W_Q, W_scales, C, M, N, K) &
                bind(C, name="q35_matmul_int4_awq")
            import :: c_int, c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(*), W_Q(*)
            real(c_float), intent(in) :: W_scales(*)
            integer(c_int32_t), intent(inout) :: C(*)
        end function q35_matmul_int4_awq

        integer(c_int) function q35_matmul_int4_fused(A, W_Q, W_scales, Out, M, N, K) &
                bind(C, name="q35_matmul_int4_fused")
            import :: c_int, c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(*), W_Q(*)
            real(c_float), intent(in) :: W_scales(*)
            real(c_float), intent(inout) :: Out(*)
        end function q35_matmul_int4_fused
    end interface

contains

    ! matmul_cuda_fortran.cuf:184-229: int32 C(M,N)
    subroutine matmul_int4_cuda(A, W_Q, W_scales, C, M, N, K_dim, stat)
        integer(int8), intent(in) :: A(:,:)
        integer(int8), intent(in) :: W_Q(:,:)
        real(real32), intent(in) :: W_scales(:)
        integer(int32), intent(out) :: C(:,:)
        integer(int32), intent(in) :: M, N, K_dim
        integer, intent(out), optional :: stat
        call q35_check(q35_matmul_int4_awq(A, W_Q, W_scales, C, M, N, K_dim), "matmul_int4_cuda", stat)
    end subroutine matmul_int4_cuda

    ! matmul_cuda_fortran.cuf:233-276: dequantized fp32 Out(M,N)
    subroutine matmul_int4_cuda_fused(A, W_Q, W_scales, Out, M, N, K_dim, stat)
        integer(int8), intent(in) :: A(:,:)
        integer(int8), intent(in) :: W_Q(:,:)
        real(real32), intent(in) :: W_scales(:)
        real(real32), intent(out) :: Out(:,:)
        integer(int32), intent(in) :: M, N, K_dim
        integer, intent(out), optional :: stat
        call q35_check(q35_matmul_int4_fused(A, W_Q, W_scales, Out, M, N, K_dim), "matmul_int4_cuda_fused", stat)
    end subroutine matmul_int4_cuda_fused

end module matmul_cuda_fortran
