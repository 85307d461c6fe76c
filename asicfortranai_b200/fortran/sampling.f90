! Drop-in replacement of module sampling (sampling.f90) over libq35.so: same module name,
! public procedure names, argument order and results (1-based token ids).  Each draw
! runs on the GPU; random_number still supplies the uniform draw, as in the reference.
! apply_temperature and softmax stay host procedures with the reference's arithmetic.
! A libq35 failure stops the program with its message (q35_status).
! Link: gfortran -c q35_status.f90 sampling.f90 && ... -L<pkg> -lq35 -Wl,-rpath,<pkg>
module sampling
    use iso_c_binding, only: c_int, c_int32_t, c_float, c_null_ptr, c_ptr
    use iso_fortran_env, only: int32, real32
    use q35_status, only: q35_check
    implicit none
    private
    public :: sample_greedy, sample_top_k, sample_top_p, sample_temperature
    public :: apply_temperature, softmax

    interface
        integer(c_int) function q35_sample_greedy(ctx, logits, vocab, token) bind(C, name="q35_sample_greedy")
            import :: c_int, c_int32_t, c_float, c_ptr
            type(c_ptr), value :: ctx
            real(c_float), intent(in) :: logits(*)
            integer(c_int32_t), value :: vocab
            integer(c_int32_t), intent(out) :: token
        end function q35_sample_greedy
        integer(c_int) function q35_sample_temperature(ctx, logits, vocab, t, u, token) &
                bind(C, name="q35_sample_temperature")
            import :: c_int, c_int32_t, c_float, c_ptr
            type(c_ptr), value :: ctx
            real(c_float), intent(in) :: logits(*)
            integer(c_int32_t), value :: vocab
            real(c_float), value :: t, u
            integer(c_int32_t), intent(out) :: token
        end function q35_sample_temperature
        integer(c_int) function q35_sample_top_k(ctx, logits, vocab, k, u, token) bind(C, name="q35_sample_top_k")
            import :: c_int, c_int32_t, c_float, c_ptr
            type(c_ptr), value :: ctx
            real(c_float), intent(in) :: logits(*)
            integer(c_int32_t), value :: vocab, k
            real(c_float), value :: u
            integer(c_int32_t), intent(out) :: token
        end function q35_sample_top_k
        integer(c_int) function q35_sample_top_p(ctx, logits, vocab, p, u, token) bind(C, name="q35_sample_top_p")
            import :: c_int, c_int32_t, c_float, c_ptr
            type(c_ptr), value :: ctx
            real(c_float), intent(in) :: logits(*)
            integer(c_int32_t), value :: vocab
            real(c_float), value :: p, u
            integer(c_int32_t), intent(out) :: token
        end function q35_sample_top_p
    end interface

contains

    ! sampling.f90:19-30
    pure subroutine apply_temperature(logits, temperature, scaled_logits, vocab_size)
        integer(int32), intent(in) :: vocab_size
        real(real32), intent(in) :: logits(vocab_size)
        real(real32), intent(in) :: temperature
        real(real32), intent(out) :: scaled_logits(vocab_size)
        if (temperature > 0.0) then
            scaled_logits = logits / temperature
        else
            scaled_logits = logits
        end if
    end subroutine apply_temperature

    ! sampling.f90:35-59
    pure subroutine softmax(logits, probs, vocab_size)
        integer(int32), intent(in) :: vocab_size
        real(real32), intent(in) :: logits(vocab_size)
        real(real32), intent(out) :: probs(vocab_size)
        real(real32) :: max_logit, sum_exp
        integer(int32) :: i
        max_logit = maxval(logits)
        sum_exp = 0.0
        do i = 1, vocab_size
            probs(i) = exp(logits(i) - max_logit)
            sum_exp = sum_exp + probs(i)
        end do
        if (sum_exp > 0.0) then
            probs = probs / sum_exp
        else
            probs = 1.0 / real(vocab_size, real32)
        end if
    end subroutine softmax

    ! a uniform draw in [0, 1) on the 24-bit grid the device uses
    real(real32) function draw()
        real(real32) :: r
        call random_number(r)
        draw = real(floor(r * 16777216.0), real32) / 16777216.0
        if (draw >= 1.0) draw = 0.0
    end function draw

    ! sampling.f90:64-83
    function sample_greedy(logits, vocab_size) result(token_id)
        integer(int32), intent(in) :: vocab_size
        real(real32), intent(in) :: logits(vocab_size)
        integer(int32) :: token_id
        call q35_check(q35_sample_greedy(c_null_ptr, logits, vocab_size, token_id), "sample_greedy")
    end function sample_greedy

    ! sampling.f90:88-118
    function sample_temperature(logits, vocab_size, temperature) result(token_id)
        integer(int32), intent(in) :: vocab_size
        real(real32), intent(in) :: logits(vocab_size)
        real(real32), intent(in) :: temperature
        integer(int32) :: token_id
        call q35_check(q35_sample_temperature(c_null_ptr, logits, vocab_size, temperature, draw(), token_id), &
                       "sample_temperature")
    end function sample_temperature

    ! sampling.f90:123-176
    function sample_top_k(logits, vocab_size, k) result(token_id)
        integer(int32), intent(in) :: vocab_size, k
        real(real32), intent(in) :: logits(vocab_size)
        integer(int32) :: token_id
        call q35_check(q35_sample_top_k(c_null_ptr, logits, vocab_size, k, draw(), token_id), "sample_top_k")
    end function sample_top_k

    ! sampling.f90:181-259
    function sample_top_p(logits, vocab_size, p) result(token_id)
        integer(int32), intent(in) :: vocab_size
        real(real32), intent(in) :: logits(vocab_size), p
        integer(int32) :: token_id
        call q35_check(q35_sample_top_p(c_null_ptr, logits, vocab_size, p, draw(), token_id), "sample_top_p")
    end function sample_top_p

end module sampling
