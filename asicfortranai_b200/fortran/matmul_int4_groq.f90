! Drop-in replacement of module matmul_int4_groq (matmul_int4_groq.f90) over libq35.so.
! The reference passes M, N, K_dim by reference; the C entry points take them by value.
! Each procedure takes an optional stat= argument; without it a failure stops the program
! with libq35's message (q35_status).
! Link: gfortran -c q35_status.f90 matmul_int4_groq.f90 && ... -L<pkg> -lq35 -Wl,-rpath,<pkg>
module matmul_int4_groq
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float
    use iso_fortran_env, only: int8, int32, real32
    use q35_status, only: q35_check
    implicit none
    private
    public :: matmul_int4_awq, dequantize_output

    interface
        integer(c_int) function q35_matmul_int4_awq(A, W_Q, W_scales, C, M, N, K) &
                bind(C, name="q35_matmul_int4_awq")
            import :: c_int, c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(M, K), W_Q(K/2, N)
            real(c_float), intent(in) :: W_scales(N)
            integer(c_int32_t), intent(inout) :: C(M, N)
        end function q35_matmul_int4_awq

        integer(c_int) function q35_dequantize_output(C, W_scales, Out, M, N) &
                bind(C, name="q35_dequantize_output")
            import :: c_int, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N
            integer(c_int32_t), intent(in) :: C(M, N)
            real(c_float), intent(in) :: W_scales(N)
            real(c_float), intent(inout) :: Out(M, N)
        end function q35_dequantize_output
    end interface

contains

    ! matmul_int4_groq.f90:19-54
    subroutine matmul_int4_awq(A, W_Q, W_scales, C, M, N, K_dim, stat)
        integer(int32), intent(in) :: M, N, K_dim
        integer(int8), intent(in) :: A(M, K_dim)
        integer(int8), intent(in) :: W_Q(K_dim/2, N)
        real(real32), intent(in) :: W_scales(N)
        integer(int32), intent(out) :: C(M, N)
        integer, intent(out), optional :: stat
        call q35_check(q35_matmul_int4_awq(A, W_Q, W_scales, C, M, N, K_dim), "matmul_int4_awq", stat)
    end subroutine matmul_int4_awq

    ! matmul_int4_groq.f90:58-69
    subroutine dequantize_output(C, W_scales, Out, M, N, stat)
        integer(int32), intent(in) :: M, N
        integer(int32), intent(in) :: C(M, N)
        real(real32), intent(in) :: W_scales(N)
        real(real32), intent(out) :: Out(M, N)
        integer, intent(out), optional :: stat
        call q35_check(q35_dequantize_output(C, W_scales, Out, M, N), "dequantize_output", stat)
    end subroutine dequantize_output

end module matmul_int4_groq
